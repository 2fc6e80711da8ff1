"""PyTorch binding of the B200 ZipServ library (ctypes over the C ABI).

Drop-in for ``zipserv_vllm.runtime`` (integrations/vllm/zipserv_vllm/runtime.py):
same names (``BUFFER_NAMES``, ``PackedWeight``, ``compress``, ``linear``,
``decompress``, ``require_fp32_partials``, the ``zipserv_vllm::linear`` custom
op and its fake), same argument meaning and the same errors for the same
invalid inputs. What differs is below the C ABI: sm_100a kernels, an
in-kernel Split-K reduction (no workspace is allocated or written) and a
packer that is byte-identical to the reference's.

The library is the in-tree ``_lib/libzipserv_b200.so`` unless
``ZIPSERV_LIBRARY`` names another ABI-2 library. There is no CPU fallback:
GPU entry points raise when the native library or CUDA is unavailable.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path

import torch
from torch import Tensor

BUFFER_NAMES = ("sm", "rare", "bitmap1", "bitmap2", "bitmap3", "medium", "global")
DEFAULT_LIBRARY = Path(__file__).resolve().parent / "_lib" / "libzipserv_b200.so"
INT32_MAX = 2**31 - 1


class _NativePacked(ctypes.Structure):
    # include/zipserv_bridge.h: struct Packed
    _fields_ = [
        ("buffers", ctypes.c_void_p * 7),
        ("lengths", ctypes.c_uint64 * 7),
        ("m", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("max_common", ctypes.c_int32),
        ("max_rare", ctypes.c_int32),
        ("start_exp", ctypes.c_int32),
    ]


def library_path() -> Path:
    override = os.environ.get("ZIPSERV_LIBRARY")
    return Path(override) if override else DEFAULT_LIBRARY


@lru_cache(maxsize=1)
def _library() -> ctypes.CDLL:
    path = library_path()
    if not path.is_file():
        raise RuntimeError(
            f"Build the ZipServ bridge (python -m zipserv_asplos26_b200.build) or set "
            f"ZIPSERV_LIBRARY to its shared library; {path} does not exist"
        )
    lib = ctypes.CDLL(str(path))
    ptr, integer = ctypes.c_void_p, ctypes.c_int
    lib.zipserv_abi_version.restype = integer
    if lib.zipserv_abi_version() != 2:
        raise RuntimeError("Unsupported ZipServ bridge ABI")
    lib.zipserv_error.restype = ctypes.c_char_p
    lib.zipserv_compress.argtypes = [ptr, integer, integer, ctypes.POINTER(_NativePacked)]
    lib.zipserv_compress.restype = integer
    lib.zipserv_free.argtypes = [ctypes.POINTER(_NativePacked)]
    lib.zipserv_free.restype = None
    if hasattr(lib, "zipserv_mm") and hasattr(lib, "zipserv_decode"):
        lib.zipserv_mm.argtypes = [ptr] * 8 + [integer] * 3 + [ptr] * 2 + [integer] * 3 + [ptr, integer]
        lib.zipserv_mm.restype = integer
        if hasattr(lib, "zipserv_mm_fp32"):
            lib.zipserv_mm_fp32.argtypes = lib.zipserv_mm.argtypes
            lib.zipserv_mm_fp32.restype = integer
        lib.zipserv_decode.argtypes = [ptr] * 8 + [integer] * 3 + [ptr] + [integer] * 2
        lib.zipserv_decode.restype = integer
    if hasattr(lib, "zipserv_mm_kparts"):
        lib.zipserv_mm_kparts.argtypes = [ptr] * 8 + [integer] * 3 + [ptr] * 2 + [integer] * 4
        lib.zipserv_mm_kparts.restype = integer
        lib.zipserv_mm_plan.argtypes = [integer] * 3
        lib.zipserv_mm_plan.restype = integer
        lib.zipserv_device_flags.argtypes = [ctypes.POINTER(ctypes.c_uint), integer]
        lib.zipserv_device_flags.restype = integer
    if hasattr(lib, "zipserv_mm_ws"):
        u64 = ctypes.c_uint64
        lib.zipserv_mm_ws.argtypes = ([ptr] * 8 + [integer] * 3 + [ptr] * 2 + [integer] * 4 +
                                      [ptr, u64, ptr, u64])
        lib.zipserv_mm_ws.restype = integer
        lib.zipserv_mm_workspace_size.argtypes = [integer] * 4 + [ctypes.POINTER(u64)] * 2
        lib.zipserv_mm_workspace_size.restype = integer
    return lib


def _cuda_library() -> ctypes.CDLL:
    lib = _library()
    if not hasattr(lib, "zipserv_mm") or not hasattr(lib, "zipserv_decode"):
        raise RuntimeError(
            "This ZipServ library has no CUDA support; rebuild with --arch for GPU execution"
        )
    return lib


def require_fp32_partials() -> None:
    """Reject old ABI-2 libraries before opting into the FP32 scratch symbol."""
    if not hasattr(_cuda_library(), "zipserv_mm_fp32"):
        raise RuntimeError(
            "FP32 partials require a bridge exporting zipserv_mm_fp32; rebuild the CUDA library"
        )


def _free_packed(lib: ctypes.CDLL, native: _NativePacked) -> None:
    lib.zipserv_free(ctypes.byref(native))


class _NativeBufferOwner:
    """Release native allocations after the last tensor storage view is gone."""

    __slots__ = ("__weakref__", "_finalizer")

    def __init__(self, lib: ctypes.CDLL, native: _NativePacked) -> None:
        self._finalizer = weakref.finalize(self, _free_packed, lib, native)
        # Live tensor storage is not freed during interpreter shutdown; the OS
        # reclaims what is still reachable at exit.
        self._finalizer.atexit = False


def _check(status: int) -> None:
    if status:
        message = _library().zipserv_error().decode("utf-8", errors="replace")
        raise RuntimeError(f"ZipServ native call failed ({status}): {message}")


@dataclass(frozen=True)
class PackedWeight:
    """Seven owned byte buffers and the native BF16 decoding metadata."""

    buffers: tuple[Tensor, ...]
    m: int
    k: int
    max_common: int
    max_rare: int
    start_exp: int

    @property
    def storage_bytes(self) -> int:
        """Logical payload and index size, excluding allocator padding."""
        return sum(buffer.numel() for buffer in self.buffers)

    def to(self, device: torch.device | str) -> "PackedWeight":
        """Transfer packed bytes without changing their representation.

        On a GPU the seven streams share one allocation, each at a 256-byte
        aligned offset: the three equally sized bitmap planes then sit at equal
        distances, which lets the kernels fetch all three with one tensor copy.
        """
        device = torch.device(device)
        if device.type != "cuda":
            buffers = tuple(buffer.to(device) for buffer in self.buffers)
        else:
            offsets, total = [], 0
            for buffer in self.buffers:
                offsets.append(total)
                total += (buffer.numel() + 255) // 256 * 256
            storage = torch.empty(max(total, 256), dtype=torch.uint8, device=device)
            views = []
            for buffer, offset in zip(self.buffers, offsets, strict=True):
                view = storage[offset:offset + buffer.numel()]
                view.copy_(buffer)
                views.append(view)
            buffers = tuple(views)
        return PackedWeight(
            buffers, self.m, self.k, self.max_common, self.max_rare, self.start_exp,
        )


def compress(weight: Tensor) -> PackedWeight:
    """Pack CPU BF16 bits; the tensors share the native buffers without a copy."""
    if weight.device.type != "cpu" or weight.dtype != torch.bfloat16 or weight.ndim != 2:
        raise ValueError("ZipServ compression requires a two-dimensional CPU BF16 tensor")
    m, k = weight.shape
    if m <= 0 or k <= 0 or m % 64 or k % 64 or m * k > 2**31 - 4097:
        raise ValueError("ZipServ requires positive, 64-aligned dimensions and int32 offsets")
    weight = weight.contiguous()
    native = _NativePacked()
    lib = _library()
    _check(lib.zipserv_compress(weight.data_ptr(), m, k, ctypes.byref(native)))
    try:
        owner = _NativeBufferOwner(lib, native)
    except BaseException:
        lib.zipserv_free(ctypes.byref(native))
        raise
    buffers = []
    for pointer, length in zip(native.buffers, native.lengths, strict=True):
        if not length:
            buffers.append(torch.empty(0, dtype=torch.uint8))
            continue
        view = (ctypes.c_uint8 * length).from_address(pointer)
        # frombuffer keeps this buffer object alive for the storage's lifetime,
        # and the buffer object keeps the owner (and so the allocation) alive.
        view._zipserv_owner = owner
        buffers.append(torch.frombuffer(view, dtype=torch.uint8))
    return PackedWeight(tuple(buffers), native.m, native.k, native.max_common,
                        native.max_rare, native.start_exp)


def _validate_buffers(buffers: list[Tensor], device: torch.device) -> None:
    if len(buffers) != 7 or any(
        tensor.device != device or tensor.dtype != torch.uint8 or not tensor.is_contiguous()
        for tensor in buffers
    ):
        raise ValueError("All seven ZipServ byte buffers must be contiguous on the input GPU")


def _gemm_limits(m: int, n: int, k: int, split_k: int) -> None:
    if max(m * n * split_k, k * n, m * k) > INT32_MAX or (m // 64) * split_k > 65535:
        raise ValueError("ZipServ output and Split-K workspace exceed native int32 indexing")


@torch.library.custom_op("zipserv_vllm::linear", mutates_args=(), device_types="cuda")
def _linear(
    x: Tensor,
    buffers: list[Tensor],
    m: int,
    k: int,
    max_common: int,
    max_rare: int,
    start_exp: int,
    split_k: int,
    fp32_partials: bool = False,
) -> Tensor:
    if m <= 0 or k <= 0 or m % 64 or k % 64:
        raise ValueError("ZipServ linear requires positive, 64-aligned weight dimensions")
    if x.dtype != torch.bfloat16 or x.ndim < 1 or x.shape[-1] != k:
        raise ValueError("ZipServ linear requires BF16 activations with the matching input width")
    if split_k < 1 or (k // 64) % split_k:
        raise ValueError("Split-K must divide the number of 64-column weight tiles")
    _validate_buffers(buffers, x.device)
    tokens = x.numel() // k
    output_shape = (*x.shape[:-1], m)
    if tokens == 0:
        return x.new_empty(output_shape)
    n = tokens
    _gemm_limits(m, n, k, split_k)
    lib = _cuda_library()
    if fp32_partials:
        require_fp32_partials()
    native_mm = lib.zipserv_mm_fp32 if fp32_partials else lib.zipserv_mm
    with torch.cuda.device(x.device):
        flat = x.reshape(tokens, k).contiguous()
        output = x.new_empty((n, m))
        stream = torch.cuda.current_stream(x.device).cuda_stream
        # Split-K is reduced inside the kernel in FP32, so no [split_k, n, m]
        # workspace is allocated; split 1 keeps the native contract satisfied.
        _check(native_mm(stream, *(b.data_ptr() for b in buffers), max_common, max_rare,
                         start_exp, flat.data_ptr(), output.data_ptr(), m, n, k, None, 1))
        return output.reshape(output_shape)


@_linear.register_fake
def _linear_fake(
    x: Tensor,
    buffers: list[Tensor],
    m: int,
    k: int,
    max_common: int,
    max_rare: int,
    start_exp: int,
    split_k: int,
    fp32_partials: bool = False,
) -> Tensor:
    return x.new_empty((*x.shape[:-1], m))


def linear(x: Tensor, packed: PackedWeight, *, split_k: int = 1,
           partial_dtype: str = "bf16") -> Tensor:
    """y = x @ W^T with W decoded on the fly; restored weights are exact, sums are FP32."""
    if partial_dtype not in ("bf16", "fp32"):
        raise ValueError("partial_dtype must be bf16 or fp32")
    return _linear(x, list(packed.buffers), packed.m, packed.k, packed.max_common,
                   packed.max_rare, packed.start_exp, split_k, partial_dtype == "fp32")


def workspace_size(m: int, n: int, k: int, k_parts: int = 0) -> tuple[int, int]:
    """(partial bytes, counter bytes) of scratch ``linear_kparts(...,
    workspace=...)`` needs on the current GPU; (0, 0) when none."""
    part, ctr = ctypes.c_uint64(0), ctypes.c_uint64(0)
    _check(_cuda_library().zipserv_mm_workspace_size(m, n, k, k_parts, ctypes.byref(part),
                                                     ctypes.byref(ctr)))
    return int(part.value), int(ctr.value)


def linear_kparts(x: Tensor, packed: PackedWeight, k_parts: int,
                  out: Tensor | None = None,
                  workspace: tuple[Tensor, Tensor] | None = None) -> Tensor:
    """``linear`` with an explicit K partition (0 = the default schedule):
    k_parts CTAs per 128-row block. ``workspace`` = (partials, counters),
    CUDA byte tensors at least ``workspace_size`` long, the counters
    zero-filled once (calls leave them zeroed; calls must not overlap),
    replaces the library's own per-stream scratch."""
    m, k = packed.m, packed.k
    if x.dtype != torch.bfloat16 or x.shape[-1] != k:
        raise ValueError("ZipServ linear requires BF16 activations with the matching input width")
    if x.device.type != "cuda":
        raise ValueError("ZipServ linear runs on CUDA tensors only")
    _validate_buffers(list(packed.buffers), x.device)
    n = x.numel() // k
    flat = x.reshape(n, k).contiguous()
    if out is None:
        out = x.new_empty((n, m))
    if n:
        _gemm_limits(m, n, k, 1)
        lib = _cuda_library()
        stream = torch.cuda.current_stream(x.device).cuda_stream
        ptrs = [b.data_ptr() for b in packed.buffers]
        if workspace is None:
            _check(lib.zipserv_mm_kparts(stream, *ptrs, packed.max_common, packed.max_rare,
                                         packed.start_exp, flat.data_ptr(), out.data_ptr(),
                                         m, n, k, k_parts))
        else:
            partials, counters = workspace
            if partials.device != x.device or counters.device != x.device:
                raise ValueError("workspace must be on the activations' device")
            _check(lib.zipserv_mm_ws(stream, *ptrs, packed.max_common, packed.max_rare,
                                     packed.start_exp, flat.data_ptr(), out.data_ptr(), m, n, k,
                                     k_parts, partials.data_ptr(),
                                     partials.numel() * partials.element_size(),
                                     counters.data_ptr(),
                                     counters.numel() * counters.element_size()))
    return out.reshape(*x.shape[:-1], m)


def plan_kparts(m: int, n: int, k: int) -> int:
    """CTAs per 128-row block of the default schedule on the current GPU
    (at least 1; the persistent grid may also give a CTA several blocks)."""
    return int(_cuda_library().zipserv_mm_plan(m, n, k))


def device_flags(clear: bool = True) -> int:
    """Device-side failure flags (bit 0: a kernel wait timed out). Synchronises."""
    flags = ctypes.c_uint(0)
    _check(_cuda_library().zipserv_device_flags(ctypes.byref(flags), int(clear)))
    return int(flags.value)


def decompress(packed: PackedWeight, *, max_bytes: int | None = None,
               out: Tensor | None = None) -> Tensor:
    """Decode to a dense [m, k] BF16 tensor on the current CUDA stream, bit-exact."""
    if max_bytes is not None:
        if type(max_bytes) is not int or max_bytes < 0:
            raise ValueError("max_bytes must be a nonnegative integer")
        if packed.m * packed.k * 2 > max_bytes:
            raise ValueError("Decoded BF16 weight exceeds its temporary allocation budget")
    device = packed.buffers[0].device
    if device.type != "cuda":
        raise ValueError("ZipServ decompression requires packed CUDA buffers")
    _validate_buffers(list(packed.buffers), device)
    lib = _cuda_library()
    with torch.cuda.device(device):
        if out is None:
            out = torch.empty((packed.m, packed.k), dtype=torch.bfloat16, device=device)
        _check(lib.zipserv_decode(torch.cuda.current_stream(device).cuda_stream,
                                  *(b.data_ptr() for b in packed.buffers), packed.max_common,
                                  packed.max_rare, packed.start_exp, out.data_ptr(),
                                  packed.m, packed.k))
    return out
