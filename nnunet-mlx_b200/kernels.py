"""Torch-tensor wrappers around the C ABI: the device operations of the inference path.

PyTorch only owns device memory and provides the current stream; every
operation here is one call into ``_nnb.so``.  Tensors must be contiguous
float32 CUDA tensors (channels-last activations ``(B, D, H, W, C)``).

Reference counterparts: ``instance_norm`` (reference
``kernels/metal_native_norm.py:92-168``), ``single_channel_conv3d``
(``kernels/metal_single_channel_conv.py:75-97``) and ``normalized_labels``
(``kernels/metal_normalized_labels.py:57-98``), plus the MLX ``conv3d`` /
``matmul`` calls of ``model/network.py``.
"""

from __future__ import annotations

import ctypes
import math
import threading
from dataclasses import dataclass, field

import numpy as np
import torch

from nnunet_mlx_b200 import _native
from nnunet_mlx_b200.errors import ContractError


class _Profile:
    """Optional CUDA-event timing of every device call (used by ``bench.py`` over its timed region).

    When enabled, each wrapper records an event pair on the current stream and
    the algorithmic FLOPs / bytes of the call; ``launches`` counts kernel
    launches of this library.
    """

    def __init__(self) -> None:
        self.active = False
        self.reset()

    def reset(self) -> None:
        self.records = []
        self.launches = 0

    def enable(self, on: bool) -> None:
        self.active = on

    def start(self, name: str, flops: float = 0.0, nbytes: float = 0.0, launches: int = 1, detail=None):
        if not self.active:
            return None
        event = torch.cuda.Event(enable_timing=True)
        event.record()
        return name, event, flops, nbytes, launches, detail() if callable(detail) else detail

    def stop(self, token) -> None:
        if token is None:
            return
        event = torch.cuda.Event(enable_timing=True)
        event.record()
        self.records.append((token, event))
        self.launches += token[4]

    def trace(self) -> list[dict]:
        """Every recorded call in order: name, detail, milliseconds, FLOPs, bytes."""
        return [{"name": name, "detail": detail, "ms": e0.elapsed_time(e1), "flops": flops, "bytes": nbytes}
                for (name, e0, flops, nbytes, _, detail), e1 in self.records]

    def summary(self) -> dict:
        out: dict[str, dict] = {}
        for (name, e0, flops, nbytes, _, _), e1 in self.records:
            item = out.setdefault(name, {"calls": 0, "seconds": 0.0, "flops": 0.0, "bytes": 0.0})
            item["calls"] += 1
            item["seconds"] += e0.elapsed_time(e1) / 1e3
            item["flops"] += flops
            item["bytes"] += nbytes
        total = sum(v["seconds"] for v in out.values()) or 1.0
        for item in out.values():
            item["share"] = item["seconds"] / total
        return out


PROFILE = _Profile()


@dataclass(frozen=True)
class Lazy:
    """An activation as stored: raw values plus the pending instance-norm affine.

    ``value = act(raw * scale[b, c] + shift[b, c])`` where ``act`` is LeakyReLU
    when ``leaky`` is set; ``scale is None`` means the raw tensor is final.
    """

    raw: torch.Tensor
    scale: torch.Tensor | None = None
    shift: torch.Tensor | None = None
    leaky: bool = False
    # tensor-core operands derived from this activation, by precision (see prepare_operand)
    prepared: dict = field(default_factory=dict, compare=False, repr=False)

    @property
    def channels(self) -> int:
        return int(self.raw.shape[-1])

    @property
    def spatial(self) -> tuple[int, int, int]:
        return tuple(int(s) for s in self.raw.shape[1:4])

    def segment(self) -> _native.Segment:
        _check_tensor(self.raw, "activation")
        if self.scale is not None:
            _check_tensor(self.scale, "scale")
            _check_tensor(self.shift, "shift")
        return _native.Segment(self.raw.data_ptr(),
                               0 if self.scale is None else self.scale.data_ptr(),
                               0 if self.shift is None else self.shift.data_ptr(),
                               self.channels, 1 if self.leaky else 0)


_STAGING: dict = {}
_STAGING_LOCK = threading.Lock()


def to_host(t: torch.Tensor) -> np.ndarray:
    """A device tensor as a fresh host numpy array, through a cached page-locked staging buffer.

    A device-to-pageable copy runs at a few GB/s (the driver stages it through
    small page-locked buffers of its own: ~0.33 s for the 715 MB logits of a
    768^2 x 101 CT on B200); the copy into a page-locked buffer runs at the
    link's rate (~13 ms) and the multithreaded host copy into the result adds
    the rest.  The staging buffer (the largest size seen, per device) lives for
    the process; pinning it is a one-time cost.
    """
    if not t.is_cuda:
        return t.numpy()
    t = t.contiguous()
    nbytes = t.numel() * t.element_size()
    with _STAGING_LOCK:
        buf = _STAGING.get(t.device.index)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 16), dtype=torch.uint8, pin_memory=True)
            _STAGING[t.device.index] = buf
        staging = buf[:nbytes].view(t.dtype).view(t.shape)
        staging.copy_(t)  # waits for the stream's pending work, then copies at the link's rate
        out = torch.empty(t.shape, dtype=t.dtype)
        out.copy_(staging)  # parallel host copy into fresh pageable memory
    return out.numpy()


def _check_tensor(t: torch.Tensor | None, name: str) -> None:
    if t is None or not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
        raise ContractError(f"{name} must be a contiguous float32 CUDA tensor")


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _operand_floats(precision: int) -> int:
    """32-bit words per channel of a prepared operand (fp16 pair: 1, TF32 pair: 2, TF32: 1, bf16: 1)."""
    return 2 if precision == _native.PREC_FP32_TF32 else 1


def prepare_operand(x: Lazy, precision: int, slope: float) -> Lazy:
    """The tensor-core operand of ``x`` (affine + LeakyReLU applied once, in the precision's format).

    Cached on ``x`` so an activation read by two convolutions (an encoder output
    and its skip connection) is prepared once.
    """
    cached = x.prepared.get(precision)
    if cached is not None:
        return cached
    halves = _operand_floats(precision)
    out = torch.empty((*x.raw.shape[:-1], halves * x.channels), dtype=torch.float32, device=x.raw.device)
    seg = x.segment()
    voxels = math.prod(x.spatial)
    token = PROFILE.start("prepare_operand", 0.0, 4.0 * x.raw.numel() * (1 + halves))
    _native.check(_native.load().nnb_prepare_operand(ctypes.byref(seg), int(x.raw.shape[0]), voxels, float(slope),
                                                     int(precision), out.data_ptr(), _stream()), "prepare_operand")
    PROFILE.stop(token)
    # the prepared tensor's segment: channels are the logical channel count
    operand = _Prepared(out, x.channels)
    x.prepared[precision] = operand
    return operand


class _Prepared(Lazy):
    """A prepared operand: ``raw`` holds the format's 32-bit words (1 or 2 per logical channel) per voxel."""

    def __init__(self, raw: torch.Tensor, logical_channels: int) -> None:
        super().__init__(raw)
        object.__setattr__(self, "logical_channels", logical_channels)

    @property
    def channels(self) -> int:
        return self.logical_channels


class OperandOnly(Lazy):
    """An activation that exists only as its tensor-core operand for one precision.

    ``raw`` is the operand buffer of ``precision`` (fp16 pair, bf16 or TF32: 4
    bytes per channel, so it has the activation's shape as float32 words) and
    is not a float32 activation: ``segment()`` refuses, and only consumers that
    take the prepared operand (tensor-core convolutions in that precision) can
    read it.
    """

    def __init__(self, operand: torch.Tensor, precision: int = _native.PREC_FP32) -> None:
        super().__init__(operand)
        object.__setattr__(self, "precision", precision)
        self.prepared[precision] = _Prepared(operand, int(operand.shape[-1]))

    def segment(self) -> _native.Segment:
        raise ContractError(f"this activation exists only as a precision-{self.precision} tensor-core operand")


def _query_segment(item: Lazy) -> _native.Segment:
    """The segment a shape query sees: an operand-only activation shows its prepared operand."""
    if isinstance(item, OperandOnly):
        seg = item.prepared[item.precision].segment()
        seg.prepared = 1
        return seg
    return item.segment()


def operand_range_events(reset: bool = False) -> int:
    """Activations found outside the fp16-pair operand's range since the last reset (synchronises)."""
    count = int(_native.load().nnb_operand_range_events(1 if reset else 0))
    if count < 0:
        _native.check(int(count), "operand_range_events")
    return count


def packed_bytes(cout: int, kvol: int, cin: int, precision: int) -> int:
    return int(_native.load().nnb_conv3d_packed_bytes(cout, kvol, cin, precision))


def pack_weights(weight: torch.Tensor, precision: int) -> torch.Tensor | None:
    """Tensor-core weight image of a converted-layout ``(C_out, kD, kH, kW, C_in)`` weight.

    Returns ``None`` when the layer is outside the tensor-core envelope (it
    then runs on the CUDA-core kernel).
    """
    if precision not in _native.TENSOR_PRECISIONS:
        return None
    _check_tensor(weight, "weight")
    cout, cin = int(weight.shape[0]), int(weight.shape[-1])
    kvol = int(math.prod(weight.shape[1:-1]))
    nbytes = packed_bytes(cout, kvol, cin, precision)
    if nbytes <= 0 or cout % 16 != 0:
        return None
    # over-allocate so the image can start on a 1024-byte boundary
    storage = torch.empty(nbytes + 1024, dtype=torch.uint8, device=weight.device)
    offset = (-storage.data_ptr()) % 1024
    image = storage[offset:offset + nbytes]
    _native.check(_native.load().nnb_conv3d_pack(weight.data_ptr(), cout, kvol, cin, precision,
                                                 image.data_ptr(), _stream()), "conv3d_pack")
    return image


def _zstream_segments(inputs: list[Lazy], precision: int, slope: float, args) -> None:
    """Segments of a convolution whose tensor-core kernel also accepts raw activations.

    The kernel's in-shared-memory preparation competes with its MMAs for
    shared-memory bandwidth, which pays only for a single 32-channel input
    that nothing else prepares: such an input is passed raw.  Every other
    segment is passed prepared (reusing an operand already prepared for
    another consumer).
    """
    raw_ok = len(inputs) == 1 and inputs[0].channels == 32
    for index, item in enumerate(inputs):
        cached = item.prepared.get(precision)
        if cached is None and raw_ok:
            continue  # keeps the raw lazy segment set by the caller
        seg = (cached if cached is not None else prepare_operand(item, precision, slope)).segment()
        seg.prepared = 1
        args.seg[index] = seg


def conv3d(inputs: list[Lazy], weight: torch.Tensor, *, kernel, stride, pad, cout: int,
           packed: torch.Tensor | None = None, bias: torch.Tensor | None = None,
           precision: int = _native.PREC_FP32, slope: float = 0.01, stats: bool = True):
    """Convolution of the channel concatenation of ``inputs``; returns ``(out, partials)``."""
    if not 1 <= len(inputs) <= 2:
        raise ContractError("conv3d takes one or two input segments")
    first = inputs[0]
    batch = int(first.raw.shape[0])
    in_dims = first.spatial
    for item in inputs[1:]:
        if item.spatial != in_dims or int(item.raw.shape[0]) != batch:
            raise ContractError("concatenated convolution inputs must share batch and spatial shape")
    out_dims = tuple((i + 2 * p - k) // s + 1 for i, p, k, s in zip(in_dims, pad, kernel, stride))
    if min(out_dims) < 1:
        raise ContractError(f"convolution output would be empty for input {in_dims}")
    device = first.raw.device
    out = torch.empty((batch, *out_dims, cout), dtype=torch.float32, device=device)
    args = _native.Conv3dArgs()
    args.batch = batch
    args.in_dims = _native.dims3(in_dims)
    args.out_dims = _native.dims3(out_dims)
    args.kernel = _native.dims3(kernel)
    args.stride = _native.dims3(stride)
    args.pad = _native.dims3(pad)
    args.num_segments = len(inputs)
    for index, item in enumerate(inputs):
        args.seg[index] = _query_segment(item)
    args.slope = float(slope)
    args.cout = int(cout)
    _check_tensor(weight, "weight")
    args.weight = weight.data_ptr()
    args.packed = _ptr(packed)
    args.bias = _ptr(bias)
    args.out = out.data_ptr()
    args.precision = int(precision)
    cin = sum(item.channels for item in inputs)
    tensor_cores = (packed is not None and precision in _native.TENSOR_PRECISIONS
                    and all(item.channels % 32 == 0 for item in inputs) and cout % 16 == 0)
    if tensor_cores and _native.load().nnb_conv3d_raw_operands(ctypes.byref(args)) == 1:
        args.operand_format = 2  # raw lazy or prepared segments (z-streaming kernel)
        _zstream_segments(inputs, precision, slope, args)
    elif tensor_cores:
        for index, item in enumerate(inputs):
            args.seg[index] = prepare_operand(item, precision, slope).segment()
        args.operand_format = 1
    else:
        args.operand_format = 0
    partials = None
    if stats:
        tiles = int(_native.load().nnb_conv3d_partial_tiles(ctypes.byref(args)))
        if tiles < 1:
            _native.check(tiles or -1, "conv3d_partial_tiles")
        partials = torch.empty((batch, cout, tiles, 3), dtype=torch.float32, device=device)
        args.partials = partials.data_ptr()
    flops = 2.0 * batch * math.prod(out_dims) * cout * cin * math.prod(kernel)
    token = PROFILE.start("conv3d_tc" if tensor_cores else "conv3d_simt", flops,
                          4.0 * (out.numel() + sum(item.raw.numel() for item in inputs)),
                          detail=lambda: (f"{batch}x{'x'.join(map(str, in_dims))} "
                                          f"{'+'.join(str(i.channels) for i in inputs)}->{cout} "
                                          f"k{'x'.join(map(str, kernel))} s{'x'.join(map(str, stride))} "
                                          f"{conv3d_kernel_name(args)}"))
    _native.check(_native.load().nnb_conv3d(ctypes.byref(args), _stream()), "conv3d")
    PROFILE.stop(token)
    return out, partials


def conv3d_kernel_name(args) -> str:
    """Name of the kernel ``nnb_conv3d`` launches for ``args`` (box, halo, z-streaming or CUDA-core)."""
    mode = int(_native.load().nnb_conv3d_kernel_mode(ctypes.byref(args)))
    if mode < 0:
        _native.check(mode, "conv3d_kernel_mode")
    return _native.KERNEL_MODES[mode]


def instance_norm_finalize(partials: torch.Tensor, gamma: torch.Tensor | None, beta: torch.Tensor | None,
                           eps: float):
    """Per-(sample, channel) ``(scale, shift)`` from ``(B, C, tiles, 3)`` (sum, M2, n) partials."""
    batch, channels, tiles, _ = partials.shape
    scale = torch.empty((batch, channels), dtype=torch.float32, device=partials.device)
    shift = torch.empty_like(scale)
    token = PROFILE.start("instance_norm_finalize", 0.0, partials.numel() * 4.0)
    _native.check(_native.load().nnb_instance_norm_finalize(
        partials.data_ptr(), batch, tiles, channels, _ptr(gamma), _ptr(beta), float(eps),
        scale.data_ptr(), shift.data_ptr(), _stream()), "instance_norm_finalize")
    PROFILE.stop(token)
    return scale, shift


def conv3d_norm_static(inputs: list[Lazy], weight: torch.Tensor, *, kernel, stride, pad, cout: int,
                       gamma: torch.Tensor | None, beta: torch.Tensor | None, eps: float,
                       packed: torch.Tensor | None = None, precision: int = _native.PREC_FP32,
                       slope: float = 0.01):
    """``conv3d`` + ``instance_norm_finalize`` through ``nnb_conv3d_norm_static``.

    The native call allocates nothing: its partial statistics live in the
    library's fixed device scratch (``NNB_STATIC_PARTIALS_FLOATS`` floats, one
    per device, so calls on one device must not overlap).  Returns
    ``(out, scale, shift)``; a layer whose partials exceed the scratch raises
    ``ContractError``.  Outputs (and a prepared operand where the tensor-core
    path does not read the raw activation) are allocated here by torch,
    outside the native call.
    """
    first = inputs[0]
    batch = int(first.raw.shape[0])
    in_dims = first.spatial
    for item in inputs[1:]:
        if item.spatial != in_dims or int(item.raw.shape[0]) != batch:
            raise ContractError("concatenated convolution inputs must share batch and spatial shape")
    out_dims = tuple((i + 2 * p - k) // s + 1 for i, p, k, s in zip(in_dims, pad, kernel, stride))
    if min(out_dims) < 1:
        raise ContractError(f"convolution output would be empty for input {in_dims}")
    device = first.raw.device
    _check_tensor(weight, "weight")
    out = torch.empty((batch, *out_dims, cout), dtype=torch.float32, device=device)
    scale = torch.empty((batch, cout), dtype=torch.float32, device=device)
    shift = torch.empty_like(scale)
    tensor_cores = (packed is not None and precision in _native.TENSOR_PRECISIONS
                    and all(item.channels % 32 == 0 for item in inputs) and cout % 16 == 0)
    args = _native.Conv3dArgs()
    args.batch = batch
    args.in_dims = _native.dims3(in_dims)
    args.out_dims = _native.dims3(out_dims)
    args.kernel = _native.dims3(kernel)
    args.stride = _native.dims3(stride)
    args.pad = _native.dims3(pad)
    args.num_segments = len(inputs)
    args.precision = int(precision)
    args.cout = int(cout)
    for index, item in enumerate(inputs):
        args.seg[index] = _query_segment(item)
    args.slope = float(slope)
    raw = tensor_cores and _native.load().nnb_conv3d_raw_operands(ctypes.byref(args)) == 1
    if raw:
        _zstream_segments(inputs, precision, slope, args)
    if tensor_cores and not raw:
        for index, item in enumerate(inputs):
            args.seg[index] = prepare_operand(item, precision, slope).segment()
    args.cout = int(cout)
    args.weight = weight.data_ptr()
    args.packed = _ptr(packed) if tensor_cores else 0
    args.bias = 0
    args.out = out.data_ptr()
    args.partials = 0
    args.operand_format = (2 if raw else 1) if tensor_cores else 0
    _native.check(_native.load().nnb_conv3d_norm_static(
        ctypes.byref(args), _ptr(gamma), _ptr(beta), float(eps), scale.data_ptr(), shift.data_ptr(), _stream()),
        "conv3d_norm_static")
    return out, scale, shift


def pack_transposed_weights(weight: torch.Tensor, precision: int) -> torch.Tensor | None:
    """Tensor-core image of a stride == kernel transposed-convolution weight ``(C_out, kD, kH, kW, C_in)``."""
    if precision not in _native.TENSOR_PRECISIONS:
        return None
    _check_tensor(weight, "weight")
    cout, cin = int(weight.shape[0]), int(weight.shape[-1])
    ktaps = int(math.prod(weight.shape[1:-1]))
    nbytes = int(_native.load().nnb_conv_transpose3d_packed_bytes(cout, ktaps, cin, precision))
    if nbytes <= 0:
        return None
    storage = torch.empty(nbytes + 1024, dtype=torch.uint8, device=weight.device)
    offset = (-storage.data_ptr()) % 1024
    image = storage[offset:offset + nbytes]
    _native.check(_native.load().nnb_conv_transpose3d_pack(weight.data_ptr(), cout, ktaps, cin, precision,
                                                           image.data_ptr(), _stream()), "conv_transpose3d_pack")
    return image


def conv_transpose3d(x: Lazy, weight: torch.Tensor, bias: torch.Tensor | None, kernel,
                     slope: float = 0.01, packed: torch.Tensor | None = None,
                     precision: int = _native.PREC_SIMT) -> torch.Tensor:
    batch = int(x.raw.shape[0])
    cout = int(weight.shape[0])
    out_dims = tuple(s * k for s, k in zip(x.spatial, kernel))
    out = torch.empty((batch, *out_dims, cout), dtype=torch.float32, device=x.raw.device)
    _check_tensor(weight, "weight")
    tensor_cores = (packed is not None and x.channels % 32 == 0 and cout % 32 == 0
                    and precision in _native.TENSOR_PRECISIONS)
    seg = prepare_operand(x, precision, slope).segment() if tensor_cores else x.segment()
    token = PROFILE.start("conv_transpose3d_tc" if tensor_cores else "conv_transpose3d_simt",
                          2.0 * out.numel() * x.channels, 4.0 * (out.numel() + x.raw.numel()),
                          detail=lambda: (f"{batch}x{'x'.join(map(str, x.spatial))} {x.channels}->{cout} "
                                          f"up{'x'.join(map(str, kernel))}"))
    _native.check(_native.load().nnb_conv_transpose3d(
        ctypes.byref(seg), batch, _native.dims3(x.spatial), _native.dims3(kernel), float(slope),
        weight.data_ptr(), _ptr(bias), cout, _ptr(packed) if tensor_cores else 0, int(precision), out.data_ptr(),
        _stream()),
        "conv_transpose3d")
    PROFILE.stop(token)
    return out


def conv_transpose3d_operand(x: Lazy, weight: torch.Tensor, bias: torch.Tensor | None, kernel,
                             slope: float = 0.01, packed: torch.Tensor | None = None,
                             precision: int = _native.PREC_SIMT) -> Lazy:
    """The up-sampled activation for the next convolution: an ``OperandOnly`` activation on the
    fp32, bf16 and tf32 tensor-core paths (the transposed conv writes the next convolution's
    operand itself, no preparation pass), otherwise a plain ``Lazy`` of the float32 output."""
    cout = int(weight.shape[0])
    if not (packed is not None and precision in _native.OPERAND_OUTPUT_PRECISIONS and x.channels % 32 == 0
            and cout % 32 == 0):
        return Lazy(conv_transpose3d(x, weight, bias, kernel, slope, packed=packed, precision=precision))
    batch = int(x.raw.shape[0])
    out_dims = tuple(s * k for s, k in zip(x.spatial, kernel))
    out = torch.empty((batch, *out_dims, cout), dtype=torch.float32, device=x.raw.device)
    _check_tensor(weight, "weight")
    seg = prepare_operand(x, precision, slope).segment()
    token = PROFILE.start("conv_transpose3d_tc", 2.0 * out.numel() * x.channels, 4.0 * (out.numel() + x.raw.numel()),
                          detail=lambda: (f"{batch}x{'x'.join(map(str, x.spatial))} {x.channels}->{cout} "
                                          f"up{'x'.join(map(str, kernel))}"))
    _native.check(_native.load().nnb_conv_transpose3d_operand(
        ctypes.byref(seg), batch, _native.dims3(x.spatial), _native.dims3(kernel), float(slope), _ptr(bias), cout,
        packed.data_ptr(), int(precision), out.data_ptr(), _stream()), "conv_transpose3d_operand")
    PROFILE.stop(token)
    return OperandOnly(out, precision)


def residual_join(branch: Lazy, skip: Lazy, slope: float) -> torch.Tensor:
    if branch.raw.shape != skip.raw.shape:
        raise ContractError(f"residual shapes differ: {tuple(branch.raw.shape)} vs {tuple(skip.raw.shape)}")
    out = torch.empty_like(branch.raw)
    b, s = branch.segment(), skip.segment()
    voxels = math.prod(branch.spatial)
    token = PROFILE.start("residual_join", 0.0, 12.0 * out.numel())
    _native.check(_native.load().nnb_residual_join(ctypes.byref(b), ctypes.byref(s), int(branch.raw.shape[0]),
                                                   voxels, float(slope), out.data_ptr(), _stream()),
                  "residual_join")
    PROFILE.stop(token)
    return out


def gather_views(volume: torch.Tensor, offset, patch, masks: list[int], out: torch.Tensor | None = None):
    """(C, Z, Y, X) volume -> (views, *patch, C) mirrored channels-last tile batch."""
    _check_tensor(volume, "volume")
    cin = int(volume.shape[0])
    if out is None:
        out = torch.empty((len(masks), *patch, cin), dtype=torch.float32, device=volume.device)
    mask_arr = (ctypes.c_int32 * len(masks))(*masks)
    token = PROFILE.start("gather_views", 0.0, 8.0 * out.numel())
    _native.check(_native.load().nnb_gather_views(
        volume.data_ptr(), cin, _native.dims3(volume.shape[1:]), _native.dims3(offset), _native.dims3(patch),
        len(masks), mask_arr, out.data_ptr(), _stream()), "gather_views")
    PROFILE.stop(token)
    return out


def gather_tiles(volume: torch.Tensor, pad_lo, items, patch, out: torch.Tensor | None = None,
                 nonfinite: torch.Tensor | None = None):
    """Batch of ``(offset, flip_mask)`` items of a ``(C, Z, Y, X)`` volume -> ``(items, *patch, C)`` channels-last.

    Offsets are coordinates of the volume zero-padded by ``pad_lo`` before each
    axis; the padding is never materialised (zeros are loaded outside the
    volume).  ``nonfinite``: a one-element int32 device counter that every
    thread meeting a non-finite value increments (``None``: no check).
    """
    _check_tensor(volume, "volume")
    cin = int(volume.shape[0])
    n = len(items)
    if out is None or int(out.shape[0]) != n:
        out = torch.empty((n, *patch, cin), dtype=torch.float32, device=volume.device)
    offsets = (ctypes.c_int32 * (3 * n))(*(int(v) for off, _ in items for v in off))
    masks = (ctypes.c_int32 * n)(*(int(m) for _, m in items))
    if nonfinite is not None and (nonfinite.dtype != torch.int32 or not nonfinite.is_cuda):
        raise ContractError("nonfinite must be an int32 CUDA tensor")
    token = PROFILE.start("gather_views", 0.0, 8.0 * out.numel())
    _native.check(_native.load().nnb_gather_tiles(
        volume.data_ptr(), cin, _native.dims3(volume.shape[1:]), _native.dims3(pad_lo), n, offsets, masks,
        _native.dims3(patch), out.data_ptr(), _ptr(nonfinite), _stream()), "gather_tiles")
    PROFILE.stop(token)
    return out


def lazy_items(features: Lazy, lo: int, hi: int) -> Lazy:
    """Batch items ``[lo, hi)`` of a lazy activation (their raw values and per-sample affine)."""
    if lo == 0 and hi == int(features.raw.shape[0]):
        return features
    if features.scale is None:
        return Lazy(features.raw[lo:hi])
    return Lazy(features.raw[lo:hi], features.scale[lo:hi], features.shift[lo:hi], features.leaky)


def accumulate_tile(features: Lazy, masks: list[int], seg_weight: torch.Tensor, seg_bias: torch.Tensor,
                    gaussian: torch.Tensor, acc: torch.Tensor, normalizer: torch.Tensor, offset,
                    add_normalizer: bool, slope: float, view_divisor: int | None = None) -> None:
    """Fused seg head + flip-back + view mean + Gaussian-weighted add of one tile.

    ``acc`` / ``normalizer`` are float32, or float16 for the nnunet-fp16 mode
    (half window updates rounded to nearest even).  ``view_divisor``: the
    tile's full view count when ``features`` holds only some of its views
    (float32 accumulation; default: ``len(masks)``).
    """
    if view_divisor is not None and view_divisor != len(masks):
        _accumulate_views(features, masks, view_divisor, seg_weight, seg_bias, gaussian, acc, normalizer, offset,
                          add_normalizer, slope)
        return
    seg = features.segment()
    mask_arr = (ctypes.c_int32 * len(masks))(*masks)
    half = acc.dtype == torch.float16
    for t, name in ((acc, "accumulator"), (normalizer, "normalizer")):
        if not t.is_cuda or not t.is_contiguous() or t.dtype != (torch.float16 if half else torch.float32):
            raise ContractError(f"{name} must be a contiguous CUDA tensor of the accumulator dtype")
    _check_tensor(gaussian, "gaussian")
    classes = int(seg_weight.shape[0])
    pvox = math.prod(features.spatial)
    token = PROFILE.start("accumulate_tile", 2.0 * features.raw.numel() * classes,
                          4.0 * features.raw.numel() + pvox * (2 * classes + 2) * acc.element_size() + 4.0 * pvox)
    entry = _native.load().nnb_accumulate_tile_fp16 if half else _native.load().nnb_accumulate_tile
    _native.check(entry(
        ctypes.byref(seg), len(masks), mask_arr, _native.dims3(features.spatial), float(slope),
        seg_weight.data_ptr(), seg_bias.data_ptr(), classes, gaussian.data_ptr(),
        acc.data_ptr(), normalizer.data_ptr(), _native.dims3(acc.shape[:3]), _native.dims3(offset),
        1 if add_normalizer else 0, _stream()), "accumulate_tile")
    PROFILE.stop(token)


def _accumulate_views(features: Lazy, masks: list[int], view_divisor: int, seg_weight, seg_bias, gaussian, acc,
                      normalizer, offset, add_normalizer: bool, slope: float) -> None:
    seg = features.segment()
    mask_arr = (ctypes.c_int32 * len(masks))(*masks)
    if acc.dtype != torch.float32 or not acc.is_contiguous() or not normalizer.is_contiguous():
        raise ContractError("a partial-view accumulation needs contiguous float32 accumulators")
    _check_tensor(gaussian, "gaussian")
    classes = int(seg_weight.shape[0])
    pvox = math.prod(features.spatial)
    token = PROFILE.start("accumulate_tile", 2.0 * features.raw.numel() * classes,
                          4.0 * features.raw.numel() + pvox * (2 * classes + 2) * 4.0 + 4.0 * pvox)
    _native.check(_native.load().nnb_accumulate_views(
        ctypes.byref(seg), len(masks), mask_arr, int(view_divisor), _native.dims3(features.spatial), float(slope),
        seg_weight.data_ptr(), seg_bias.data_ptr(), classes, gaussian.data_ptr(), acc.data_ptr(),
        normalizer.data_ptr(), _native.dims3(acc.shape[:3]), _native.dims3(offset), 1 if add_normalizer else 0,
        _stream()), "accumulate_views")
    PROFILE.stop(token)


def fold_add_fp16(acc16: torch.Tensor, normalizer16: torch.Tensor, crop_lo, crop_dims, total16: torch.Tensor,
                  first: bool, invalid: torch.Tensor) -> None:
    """nnunet-fp16: this fold's normalised half logits over the crop into the channel-first half total."""
    classes = int(acc16.shape[-1])
    if total16.dtype != torch.float16 or tuple(total16.shape) != (classes, *crop_dims):
        raise ContractError("fold total must be float16 (C, *crop)")
    voxels = math.prod(crop_dims)
    token = PROFILE.start("fold_add_fp16", 0.0, 2.0 * voxels * (2 * classes + 1))
    _native.check(_native.load().nnb_fold_add_fp16(
        acc16.data_ptr(), normalizer16.data_ptr(), classes, _native.dims3(acc16.shape[:3]), _native.dims3(crop_lo),
        _native.dims3(crop_dims), total16.data_ptr(), 1 if first else 0, invalid.data_ptr(), _stream()),
        "fold_add_fp16")
    PROFILE.stop(token)


def fold_sum_fp16(total16: torch.Tensor, part16: torch.Tensor, invalid: torch.Tensor) -> None:
    """nnunet-fp16: ``total16 = half(total16 + part16)`` element-wise (a fold computed on another device)."""
    if (total16.dtype != torch.float16 or part16.dtype != torch.float16 or total16.shape != part16.shape
            or not total16.is_contiguous() or not part16.is_contiguous()):
        raise ContractError("fold sum needs contiguous float16 tensors of one shape")
    token = PROFILE.start("fold_sum_fp16", 0.0, 6.0 * total16.numel())
    _native.check(_native.load().nnb_fold_sum_fp16(total16.data_ptr(), part16.data_ptr(), total16.numel(),
                                                   invalid.data_ptr(), _stream()), "fold_sum_fp16")
    PROFILE.stop(token)


def fold_finalize_fp16(total16: torch.Tensor, folds: int, *, want_logits: bool = True,
                       label_dtype: torch.dtype | None = torch.uint8):
    """Fold average of the half total (in place); float32 logits of the half values, labels, invalid count."""
    classes = int(total16.shape[0])
    crop = tuple(int(v) for v in total16.shape[1:])
    voxels = math.prod(crop)
    logits = torch.empty((classes, *crop), dtype=torch.float32, device=total16.device) if want_logits else None
    labels, label_bytes = None, 1
    if label_dtype is not None:
        if label_dtype == torch.uint8:
            label_bytes = 1
        elif label_dtype in (torch.uint16, torch.int16):
            label_bytes = 2
        else:
            raise ContractError("labels must be uint8 or uint16")
        labels = torch.empty(crop, dtype=label_dtype, device=total16.device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=total16.device)
    token = PROFILE.start("fold_finalize_fp16", 0.0, voxels * (4.0 * classes + label_bytes), launches=2)
    _native.check(_native.load().nnb_fold_finalize_fp16(
        total16.data_ptr(), classes, voxels, int(folds), _ptr(logits), _ptr(labels), label_bytes, invalid.data_ptr(),
        _stream()), "fold_finalize_fp16")
    PROFILE.stop(token)
    return logits, labels, invalid


def normalize_labels(acc: torch.Tensor, normalizer: torch.Tensor, crop_lo, crop_dims, *, fold_divisor: float = 1.0,
                     want_logits: bool = True, label_dtype: torch.dtype | None = torch.uint8):
    """Normalised channel-first logits ``(C, *crop)`` and labels ``(*crop)``; invalid count tensor."""
    classes = int(acc.shape[-1])
    device = acc.device
    logits = torch.empty((classes, *crop_dims), dtype=torch.float32, device=device) if want_logits else None
    labels = None
    label_bytes = 1
    if label_dtype is not None:
        if label_dtype == torch.uint8:
            label_bytes = 1
        elif label_dtype in (torch.uint16, torch.int16):
            label_bytes = 2
        else:
            raise ContractError("labels must be uint8 or uint16")
        labels = torch.empty(tuple(crop_dims), dtype=label_dtype, device=device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=device)
    voxels = math.prod(crop_dims)
    token = PROFILE.start("normalize_labels", 0.0, 4.0 * voxels * (2 * classes + 1) + voxels * label_bytes,
                          launches=2)
    _native.check(_native.load().nnb_normalize_labels(
        acc.data_ptr(), normalizer.data_ptr(), classes, _native.dims3(acc.shape[:3]), _native.dims3(crop_lo),
        _native.dims3(crop_dims), float(fold_divisor), _ptr(logits), _ptr(labels), label_bytes,
        invalid.data_ptr(), _stream()), "normalize_labels")
    PROFILE.stop(token)
    return logits, labels, invalid


def restore_class_labels(logits: torch.Tensor, target, *, class_axis: int = 0, volume=None, crop_lo=(0, 0, 0),
                         axes=(0, 1, 2), label_dtype: torch.dtype = torch.uint16):
    """Labels of class logits resampled to ``target``, uncropped and axis-permuted, in one device pass.

    ``logits``: 4-D float32 or float16 CUDA tensor, classes on ``class_axis`` (0: ``(C, S0, S1, S2)``,
    3: ``(S0, S1, S2, C)``), any strides.  Each class is resampled to the ``target`` grid by order-1
    interpolation on the half-pixel grid with edge-clamped indices (float64, one rounding to the logits'
    dtype); the label is the first class with the largest value.  The ``target``-sized crop is placed at
    ``crop_lo`` in a zero ``volume`` (default: ``target``) and the result is permuted so that output axis
    ``i`` is volume axis ``axes[i]``.  Returns ``(labels, invalid)``: contiguous ``label_dtype`` labels and a
    one-element int32 device count of voxels whose value was not finite (labelled all ones).
    """
    if not isinstance(logits, torch.Tensor) or not logits.is_cuda or logits.dim() != 4:
        raise ContractError("restoration requires 4-D CUDA class logits")
    if logits.dtype not in (torch.float32, torch.float16):
        raise ContractError("restoration requires float32 or float16 logits")
    if class_axis not in (0, 3, -1):
        raise ContractError("class_axis must be 0 (classes first) or 3 (classes last)")
    class_axis %= 4
    spatial_axes = [a for a in range(4) if a != class_axis]
    classes = int(logits.shape[class_axis])
    source = tuple(int(logits.shape[a]) for a in spatial_axes)
    target = tuple(int(v) for v in target)
    volume = target if volume is None else tuple(int(v) for v in volume)
    if label_dtype == torch.uint8:
        label_bytes = 1
    elif label_dtype in (torch.uint16, torch.int16):
        label_bytes = 2
    else:
        raise ContractError("labels must be uint8 or uint16")
    if len(target) != 3 or len(volume) != 3 or sorted(int(a) for a in axes) != [0, 1, 2]:
        raise ContractError("restoration needs three target and volume sizes and an axis permutation")
    labels = torch.empty(tuple(volume[int(a)] for a in axes), dtype=label_dtype, device=logits.device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=logits.device)
    args = _native.RestoreArgs()
    args.logits = logits.data_ptr()
    args.half = 1 if logits.dtype == torch.float16 else 0
    args.classes = classes
    args.source_dims = _native.dims3(source)
    args.target_dims = _native.dims3(target)
    args.class_stride = int(logits.stride(class_axis))
    args.source_strides = _native.I64x3(*(int(logits.stride(a)) for a in spatial_axes))
    args.volume_dims = _native.dims3(volume)
    args.crop_lo = _native.dims3(crop_lo)
    args.axes = _native.dims3(axes)
    args.label_bytes = label_bytes
    args.labels = labels.data_ptr()
    args.invalid_count = invalid.data_ptr()
    token = PROFILE.start("restore_class_labels", 0.0,
                          float(logits.element_size() * classes * math.prod(source) + label_bytes * labels.numel()))
    _native.check(_native.load().nnb_restore_class_labels(ctypes.byref(args), _stream()), "restore_class_labels")
    PROFILE.stop(token)
    return labels, invalid


# ---- raw-case preprocessing (reference data/preprocessing.py, kernels/metal_torch_resample.py) ----

_FILL_SWEEPS_PER_CHECK = 4
_FILL_MAX_ROUNDS = 100_000


def _require_device(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ContractError(f"{name} must be a CUDA tensor")


def _raw_case(raw: torch.Tensor, transpose) -> _native.RawCase:
    """The C descriptor of a contiguous ``(C, R0, R1, R2)`` raw case; plans axis i = raw axis ``transpose[i]``."""
    _require_device(raw, "raw case")
    dtype = str(raw.dtype).removeprefix("torch.")
    if raw.dim() != 4 or not raw.is_contiguous() or dtype not in _native.RAW_DTYPES:
        raise ContractError("raw cases must be contiguous (C, X, Y, Z) float32/float64/int16/uint8/uint16/int32")
    if sorted(int(a) for a in transpose) != [0, 1, 2]:
        raise ContractError("transpose_forward must be a permutation of (0, 1, 2)")
    case = _native.RawCase()
    case.data = raw.data_ptr()
    case.dtype = _native.RAW_DTYPES[dtype]
    case.channels = int(raw.shape[0])
    case.raw_dims = _native.dims3(raw.shape[1:])
    case.transpose = _native.dims3(transpose)
    return case


def nonzero_bounds(raw: torch.Tensor, transpose=(0, 1, 2)) -> torch.Tensor:
    """Device int32[8]: inclusive lo[3], hi[3] of the nonzero voxels in plans order, then the non-finite count."""
    case = _raw_case(raw, transpose)
    bounds = torch.empty((8,), dtype=torch.int32, device=raw.device)
    token = PROFILE.start("nonzero_bounds", 0.0, float(raw.numel() * raw.element_size()))
    _native.check(_native.load().nnb_nonzero_bounds(ctypes.byref(case), bounds.data_ptr(), _stream()),
                  "nonzero_bounds")
    PROFILE.stop(token)
    return bounds


def fill_holes(raw: torch.Tensor, transpose, crop_lo, crop_dims) -> torch.Tensor:
    """int8 crop-box state of the hole-filled nonzero mask (2 = background reached from outside the box).

    Line sweeps along the three axes repeat until a round of sweeps marks no
    voxel; each round costs one synchronisation.
    """
    case = _raw_case(raw, transpose)
    dims = tuple(int(v) for v in crop_dims)
    state = torch.empty(dims, dtype=torch.int8, device=raw.device)
    changed = torch.zeros((1,), dtype=torch.int32, device=raw.device)
    lib = _native.load()
    _native.check(lib.nnb_fill_holes_init(ctypes.byref(case), _native.dims3(crop_lo), _native.dims3(dims),
                                          state.data_ptr(), _stream()), "fill_holes_init")
    for _ in range(_FILL_MAX_ROUNDS):
        changed.zero_()
        for _ in range(_FILL_SWEEPS_PER_CHECK):
            _native.check(lib.nnb_fill_holes_sweep(state.data_ptr(), _native.dims3(dims), changed.data_ptr(),
                                                   _stream()), "fill_holes_sweep")
        if int(changed.item()) == 0:
            return state
    raise ContractError("hole filling did not converge")


def crop_labels(labels: torch.Tensor, raw: torch.Tensor, transpose, crop_lo, crop_dims,
                state: torch.Tensor) -> torch.Tensor:
    """Cropped, transposed int32 previous-stage labels; background outside the filled mask becomes -1."""
    case = _raw_case(raw, transpose)
    _require_device(labels, "previous-stage labels")
    _require_device(state, "crop mask state")
    if labels.dtype != torch.int32 or not labels.is_contiguous() or tuple(labels.shape) != (1, *raw.shape[1:]):
        raise ContractError("previous-stage labels must be contiguous int32 (1, X, Y, Z) matching the image")
    dims = tuple(int(v) for v in crop_dims)
    out = torch.empty((1, *dims), dtype=torch.int32, device=raw.device)
    _native.check(_native.load().nnb_crop_labels(labels.data_ptr(), ctypes.byref(case), _native.dims3(crop_lo),
                                                 _native.dims3(dims), state.data_ptr(), out.data_ptr(), _stream()),
                  "crop_labels")
    return out


@dataclass(frozen=True)
class ChannelNormalization:
    """One channel's plans normalisation: scheme name, mask use and CT parameters (float32-rounded)."""

    scheme: str
    use_mask: bool = False
    lower: float = 0.0
    upper: float = 0.0
    mean: float = 0.0
    divisor: float = 1.0


def crop_normalize(raw: torch.Tensor, transpose, crop_lo, crop_dims, channels: list[ChannelNormalization], *,
                   state: torch.Tensor | None = None, labels: torch.Tensor | None = None):
    """``(out, errors)``: float32 ``(C, *crop_dims)`` normalised crop and device int32[4] error counts

    (non-finite outputs, RGB range violations, empty z-score selections).
    """
    case = _raw_case(raw, transpose)
    if len(channels) != int(raw.shape[0]):
        raise ContractError("normalization schemes do not match the input channels")
    table = (_native.NormChannel * len(channels))()
    for entry, spec in zip(table, channels, strict=True):
        if spec.scheme not in _native.NORM_SCHEMES:
            raise ContractError(f"unsupported nnU-Net normalization scheme {spec.scheme!r}")
        entry.scheme = _native.NORM_SCHEMES[spec.scheme]
        entry.use_mask = 1 if spec.use_mask else 0
        entry.lower, entry.upper, entry.mean, entry.divisor = spec.lower, spec.upper, spec.mean, spec.divisor
    dims = tuple(int(v) for v in crop_dims)
    out = torch.empty((len(channels), *dims), dtype=torch.float32, device=raw.device)
    errors = torch.empty((4,), dtype=torch.int32, device=raw.device)
    lib = _native.load()
    workspace = torch.empty((int(lib.nnb_crop_normalize_workspace_bytes(len(channels))),), dtype=torch.uint8,
                            device=raw.device)
    token = PROFILE.start("crop_normalize", 0.0, float(out.numel() * (raw.element_size() + 4)))
    _native.check(lib.nnb_crop_normalize(ctypes.byref(case), _native.dims3(crop_lo), _native.dims3(dims), table,
                                         _ptr(state), _ptr(labels), workspace.data_ptr(), out.data_ptr(),
                                         errors.data_ptr(), _stream()), "crop_normalize")
    PROFILE.stop(token)
    return out, errors


def torch_resize(source: torch.Tensor, target, mode: str, *, labels: bool = False,
                 tiebreak: str = "nearest") -> torch.Tensor:
    """One pass of upstream's torch-grid resampler over a 4-D ``(C, S0, S1, S2)`` CUDA tensor (any strides).

    float32 image values or int32 labels; the result is contiguous ``(C, *target)`` of the source's dtype.
    """
    _require_device(source, "resampling source")
    if source.dim() != 4 or source.dtype != (torch.int32 if labels else torch.float32):
        raise ContractError("torch-grid resampling needs (C, X, Y, Z) float32 values or int32 labels")
    if mode not in _native.RESIZE_MODES or tiebreak not in _native.TIEBREAKS:
        raise ContractError("unsupported torch-grid interpolation mode or label tie rule")
    target = tuple(int(v) for v in target)
    if len(target) != 3 or min(target) < 1 or max(*source.shape[1:], *target) >= 2**31:
        raise ContractError("torch-grid resampling needs three positive sizes within the int32 range")
    out = torch.empty((int(source.shape[0]), *target), dtype=source.dtype, device=source.device)
    args = _native.TorchResizeArgs()
    args.source = source.data_ptr()
    args.labels = 1 if labels else 0
    args.channels = int(source.shape[0])
    args.source_dims = _native.dims3(source.shape[1:])
    args.channel_stride = int(source.stride(0))
    args.source_strides = _native.I64x3(*(int(s) for s in source.stride()[1:]))
    args.target_dims = _native.dims3(target)
    args.mode = _native.RESIZE_MODES[mode]
    args.tiebreak = _native.TIEBREAKS[tiebreak]
    args.target = out.data_ptr()
    token = PROFILE.start("torch_resize", 0.0, float(out.numel() * 4 * 2))
    _native.check(_native.load().nnb_torch_resize(ctypes.byref(args), _stream()), "torch_resize")
    PROFILE.stop(token)
    return out


def spline_resize(source: torch.Tensor, target, *, axes: int = 7, order: int = 3,
                  float64_out: bool = False) -> torch.Tensor:
    """scipy-``zoom``-equivalent spline resampling of a 4-D ``(C, S0, S1, S2)`` float32/float64 CUDA tensor.

    Axes in the bit mask ``axes`` are resampled (order 3: edge padding, cubic B-spline prefilter and
    four-tap sampling on the half-pixel grid; order 1: linear); the others must keep their size.
    Returns a contiguous ``(C, *target)`` float32 (or float64) tensor.
    """
    _require_device(source, "resampling source")
    if source.dim() != 4 or source.dtype not in (torch.float32, torch.float64):
        raise ContractError("spline resampling needs (C, X, Y, Z) float32 or float64 values")
    if order not in (1, 3):
        raise ContractError(f"spline order {order} is not supported on the device (1 or 3)")
    target = tuple(int(v) for v in target)
    if len(target) != 3 or min(target) < 1 or max(*source.shape[1:], *target) >= 2**31:
        raise ContractError("spline resampling needs three positive sizes within the int32 range")
    lib = _native.load()
    dims = _native.dims3(source.shape[1:])
    workspace = torch.empty((int(lib.nnb_spline_workspace_bytes(int(source.shape[0]), dims, axes, order)) // 8,),
                            dtype=torch.float64, device=source.device)
    out = torch.empty((int(source.shape[0]), *target), dtype=torch.float64 if float64_out else torch.float32,
                      device=source.device)
    args = _native.SplineResizeArgs()
    args.source = source.data_ptr()
    args.source_f64 = 1 if source.dtype == torch.float64 else 0
    args.channels = int(source.shape[0])
    args.source_dims = dims
    args.channel_stride = int(source.stride(0))
    args.source_strides = _native.I64x3(*(int(s) for s in source.stride()[1:]))
    args.target_dims = _native.dims3(target)
    args.axes = int(axes)
    args.order = int(order)
    args.coefficients = workspace.data_ptr()
    args.target = out.data_ptr()
    args.target_f64 = 1 if float64_out else 0
    token = PROFILE.start("spline_resize", 0.0, float(workspace.numel() * 8 * 3 + out.numel() * out.element_size()))
    _native.check(lib.nnb_spline_resize(ctypes.byref(args), _stream()), "spline_resize")
    PROFILE.stop(token)
    return out


def nearest_axis_resize(source: torch.Tensor, target) -> torch.Tensor:
    """Order-0 out-of-plane pass: contiguous float64 ``(C, S0, S1, S2)`` -> float32 ``(C, *target)``."""
    _require_device(source, "resampling source")
    if source.dim() != 4 or source.dtype != torch.float64 or not source.is_contiguous():
        raise ContractError("the out-of-plane pass needs a contiguous float64 (C, X, Y, Z) tensor")
    target = tuple(int(v) for v in target)
    out = torch.empty((int(source.shape[0]), *target), dtype=torch.float32, device=source.device)
    _native.check(_native.load().nnb_nearest_axis_resize(source.data_ptr(), int(source.shape[0]),
                                                         _native.dims3(source.shape[1:]), _native.dims3(target),
                                                         out.data_ptr(), _stream()), "nearest_axis_resize")
    return out
