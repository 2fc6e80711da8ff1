"""PyTorch binding of the B200 ZipServ library (ctypes over the C ABI).

Public surface, kept identical to the reference's runtime module
(integrations/vllm/zipserv_vllm/runtime.py:18-315) so callers of that module
can switch: ``BUFFER_NAMES``, ``PackedWeight`` (same fields), ``compress``,
``linear``, ``decompress``, ``require_fp32_partials`` and the
``zipserv_vllm::linear`` custom op with the same schema and fake. Invalid
inputs raise the same exception types with the same messages.

How this module is built (its own design, not the reference's):

* The library is described by one signature table (``_SIGNATURES``); the
  loader binds every symbol the library exports and records which optional
  entry points exist.
* A packed weight lives in one *arena*: a byte tensor that holds the seven
  TCA-TBE streams at 256-byte aligned offsets, the buffers being views of it.
  ``compress`` copies the native encoder's output into a fresh arena and
  returns the native allocation before it returns, so tensor lifetimes never
  depend on native memory. ``PackedWeight.to`` moves the arena with a single
  copy; on a GPU the three equally sized bitmap planes then sit at equal
  distances, which lets the kernels fetch all three with one tensor copy.
* ``save_packed`` / ``load_packed`` store that arena with a versioned header
  (the reference has no interchange format and packs at every load).

The library is the in-tree ``_lib/libzipserv_b200.so`` unless
``ZIPSERV_LIBRARY`` names another ABI-2 library. There is no CPU fallback:
GPU entry points raise when the native library or CUDA is unavailable.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import struct
from dataclasses import dataclass, field
from functools import lru_cache
from pathlib import Path

import torch
from torch import Tensor

BUFFER_NAMES = ("sm", "rare", "bitmap1", "bitmap2", "bitmap3", "medium", "global")
DEFAULT_LIBRARY = Path(__file__).resolve().parent / "_lib" / "libzipserv_b200.so"
INT32_MAX = 2**31 - 1
ARENA_ALIGN = 256


class _Descriptor(ctypes.Structure):
    """``struct Packed`` of include/zipserv_bridge.h (the reference's
    integrations/vllm/native/host_bridge.h:9-13 layout)."""

    _fields_ = [
        ("buffers", ctypes.c_void_p * 7),
        ("lengths", ctypes.c_uint64 * 7),
        ("m", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("max_common", ctypes.c_int32),
        ("max_rare", ctypes.c_int32),
        ("start_exp", ctypes.c_int32),
    ]


# ------------------------------------------------------------------ library
_P, _I, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
# stream, the seven buffers, max_common, max_rare, start_exp, x, y, m, n, k
_GEMM_HEAD = [_P] * 8 + [_I] * 3 + [_P, _P] + [_I] * 3
_SIGNATURES: dict[str, tuple[object, list]] = {
    "zipserv_abi_version": (_I, []),
    "zipserv_error": (ctypes.c_char_p, []),
    "zipserv_compress": (_I, [_P, _I, _I, ctypes.POINTER(_Descriptor)]),
    "zipserv_free": (None, [ctypes.POINTER(_Descriptor)]),
    # GPU entry points (absent from a CPU-only build of a bridge).
    "zipserv_mm": (_I, _GEMM_HEAD + [_P, _I]),
    "zipserv_mm_fp32": (_I, _GEMM_HEAD + [_P, _I]),
    "zipserv_decode": (_I, [_P] * 8 + [_I] * 3 + [_P, _I, _I]),
    # Extensions of this library.
    "zipserv_mm_kparts": (_I, _GEMM_HEAD + [_I]),
    "zipserv_mm_ws": (_I, _GEMM_HEAD + [_I, _P, _U64, _P, _U64]),
    "zipserv_mm_noalloc": (_I, _GEMM_HEAD + [_I]),
    "zipserv_mm_plan": (_I, [_I] * 3),
    "zipserv_mm_workspace_size": (_I, [_I] * 4 + [ctypes.POINTER(_U64)] * 2),
    "zipserv_device_flags": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "zipserv_mm_reducer_wait": (_U64, [_U64]),
    "zipserv_mm_allreduce_sizes": (_I, [_I, _I, _I, ctypes.POINTER(_U64), ctypes.POINTER(_U64)]),
    "zipserv_mm_allreduce": (_I, _GEMM_HEAD + [_I, _I, _P, _P, _P, _U64, _U64]),
    "zipserv_ipc_alloc": (_I, [_U64, ctypes.POINTER(_P)]),
    "zipserv_ipc_free": (_I, [_P]),
    "zipserv_ipc_handle": (_I, [_P, _P]),
    "zipserv_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "zipserv_ipc_close": (_I, [_P]),
    "zipserv_pack_device_scratch_bytes": (_U64, []),
    "zipserv_pack_device_plan": (_I, [_P, _P, _I, _I, _I, _P, _P, ctypes.POINTER(ctypes.c_int32)]),
    "zipserv_pack_device_encode": (_I, [_P, _P, _I, _I, _P, _P] + [_P] * 6),
}
_CORE = ("zipserv_abi_version", "zipserv_error", "zipserv_compress", "zipserv_free")
_CUDA_CORE = ("zipserv_mm", "zipserv_decode")


def library_path() -> Path:
    override = os.environ.get("ZIPSERV_LIBRARY")
    return Path(override) if override else DEFAULT_LIBRARY


def _bind(lib, name: str):
    fn = getattr(lib, name)
    fn.restype, fn.argtypes = _SIGNATURES[name][0], _SIGNATURES[name][1]
    return fn


@lru_cache(maxsize=1)
def _library() -> ctypes.CDLL:
    """Load and bind the ABI-2 library (cached; ``cache_clear`` reloads)."""
    path = library_path()
    if not path.is_file():
        raise RuntimeError(
            f"Build the ZipServ bridge (python -m zipserv_asplos26_b200.build) or set "
            f"ZIPSERV_LIBRARY to its shared library; {path} does not exist"
        )
    lib = ctypes.CDLL(str(path))
    version = getattr(lib, "zipserv_abi_version")
    version.restype, version.argtypes = _I, []
    if version() != 2:
        raise RuntimeError("Unsupported ZipServ bridge ABI")
    for name in _SIGNATURES:
        if name in _CORE or hasattr(lib, name):
            _bind(lib, name)
    return lib


def _cuda_library() -> ctypes.CDLL:
    lib = _library()
    if not all(hasattr(lib, name) for name in _CUDA_CORE):
        raise RuntimeError(
            "This ZipServ library has no CUDA support; rebuild with --arch for GPU execution"
        )
    return lib


def require_fp32_partials() -> None:
    """Reject libraries that predate the FP32 scratch entry point."""
    if not hasattr(_cuda_library(), "zipserv_mm_fp32"):
        raise RuntimeError(
            "FP32 partials require a bridge exporting zipserv_mm_fp32; rebuild the CUDA library"
        )


def _check(status: int) -> None:
    if status:
        message = _library().zipserv_error().decode("utf-8", errors="replace")
        raise RuntimeError(f"ZipServ native call failed ({status}): {message}")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# -------------------------------------------------------------------- arena
def _arena_offsets(lengths) -> tuple[list[int], int]:
    """Offsets of the seven streams in an arena and its size (each stream
    starts on an ARENA_ALIGN boundary; equal lengths give equal spacing)."""
    offsets, total = [], 0
    for n in lengths:
        offsets.append(total)
        total += -(-int(n) // ARENA_ALIGN) * ARENA_ALIGN
    return offsets, max(total, ARENA_ALIGN)


def _arena_views(arena: Tensor, lengths) -> tuple[Tensor, ...]:
    offsets, _ = _arena_offsets(lengths)
    return tuple(arena[o:o + int(n)] for o, n in zip(offsets, lengths, strict=True))


def _new_arena(lengths, device: torch.device | str = "cpu") -> tuple[Tensor, tuple[Tensor, ...]]:
    _, total = _arena_offsets(lengths)
    arena = torch.empty(total, dtype=torch.uint8, device=device)
    return arena, _arena_views(arena, lengths)


@dataclass(frozen=True)
class PackedWeight:
    """Seven TCA-TBE byte buffers and the BF16 decoding metadata.

    ``arena`` (not part of the reference's fields, optional) is the byte
    tensor the buffers are views of when they were made by this module."""

    buffers: tuple[Tensor, ...]
    m: int
    k: int
    max_common: int
    max_rare: int
    start_exp: int
    arena: Tensor | None = field(default=None, compare=False, repr=False)

    @property
    def storage_bytes(self) -> int:
        """Logical payload and index size, excluding alignment padding."""
        return sum(buffer.numel() for buffer in self.buffers)

    @property
    def lengths(self) -> tuple[int, ...]:
        return tuple(buffer.numel() for buffer in self.buffers)

    def _own_arena(self) -> Tensor | None:
        """The arena, if the buffers are still its canonical views."""
        arena = self.arena
        if arena is None:
            return None
        expected = _arena_views(arena, self.lengths)
        same = all(a.data_ptr() == b.data_ptr() and a.device == b.device
                   for a, b in zip(expected, self.buffers, strict=True) if b.numel())
        return arena if same else None

    def to(self, device: torch.device | str) -> "PackedWeight":
        """The same bytes on `device`: one arena copy (buffers not made by this
        module are first gathered into an arena)."""
        device = torch.device(device)
        arena = self._own_arena()
        if arena is None:
            arena, views = _new_arena(self.lengths, self.buffers[0].device if self.buffers else "cpu")
            for view, buffer in zip(views, self.buffers, strict=True):
                view.copy_(buffer.reshape(-1).view(torch.uint8))
        moved = arena.to(device)
        return PackedWeight(_arena_views(moved, self.lengths), self.m, self.k, self.max_common,
                            self.max_rare, self.start_exp, moved)


# ------------------------------------------------------------------ packing
def _packable_problem(weight: Tensor) -> str | None:
    if weight.device.type != "cpu" or weight.dtype != torch.bfloat16 or weight.ndim != 2:
        return "ZipServ compression requires a two-dimensional CPU BF16 tensor"
    m, k = weight.shape
    if m <= 0 or k <= 0 or m % 64 or k % 64 or m * k > 2**31 - 4097:
        return "ZipServ requires positive, 64-aligned dimensions and int32 offsets"
    return None


def _release(lib: ctypes.CDLL, descriptor: _Descriptor) -> None:
    lib.zipserv_free(ctypes.byref(descriptor))


def compress(weight: Tensor) -> PackedWeight:
    """Pack CPU BF16 bits (byte-identical to the reference encoder) into an
    arena-backed PackedWeight. The native output is freed before returning,
    also when copying it fails."""
    problem = _packable_problem(weight)
    if problem:
        raise ValueError(problem)
    m, k = weight.shape
    source = weight.contiguous()
    lib = _library()
    descriptor = _Descriptor()
    _check(lib.zipserv_compress(source.data_ptr(), m, k, ctypes.byref(descriptor)))
    try:
        lengths = [int(n) for n in descriptor.lengths]
        arena, views = _new_arena(lengths)
        for view, address, n in zip(views, descriptor.buffers, lengths, strict=True):
            if n:
                ctypes.memmove(view.data_ptr(), address, n)
        meta = (descriptor.m, descriptor.k, descriptor.max_common, descriptor.max_rare,
                descriptor.start_exp)
    finally:
        _release(lib, descriptor)
    return PackedWeight(views, *meta, arena)


def compress_device(weight: Tensor, base: int = -1) -> PackedWeight:
    """Pack a BF16 matrix that is already on a GPU, on that GPU, into an
    arena there; the bytes equal ``compress(weight.cpu())`` exactly. The
    weight is read on the current stream; the call waits once for the stream
    lengths (they depend on the data). ``base`` fixes the 7-exponent window's
    first exponent (0..249) instead of choosing the most populated one."""
    if type(base) is not int or not -1 <= base <= 249:
        raise ValueError("base must be -1 or an exponent in [0, 249]")
    if weight.device.type != "cuda" or weight.dtype != torch.bfloat16 or weight.ndim != 2:
        raise ValueError("ZipServ device compression requires a two-dimensional CUDA BF16 tensor")
    m, k = weight.shape
    if m <= 0 or k <= 0 or m % 64 or k % 64 or m * k > 2**31 - 4097:
        raise ValueError("ZipServ requires positive, 64-aligned dimensions and int32 offsets")
    lib = _cuda_library()
    if not hasattr(lib, "zipserv_pack_device_plan"):
        raise RuntimeError("This ZipServ library has no device packer")
    device = weight.device
    with torch.cuda.device(device):
        source = weight.contiguous()
        tiles = (m // 64) * (k // 64)
        offsets = torch.empty((tiles + 1) * 8, dtype=torch.uint8, device=device)
        scratch = torch.empty(int(lib.zipserv_pack_device_scratch_bytes()), dtype=torch.uint8,
                              device=device)
        info = (ctypes.c_int32 * 5)()
        stream = _stream(device)
        _check(lib.zipserv_pack_device_plan(stream, source.data_ptr(), m, k, base,
                                            offsets.data_ptr(), scratch.data_ptr(), info))
        start_exp, max_common, max_rare, sm_bytes, rare_bytes = (int(v) for v in info)
        lengths = [sm_bytes, rare_bytes, tiles * 512, tiles * 512, tiles * 512, tiles * 32,
                   (tiles + 1) * 8]
        arena, views = _new_arena(lengths, device)
        views[6].copy_(offsets)
        _check(lib.zipserv_pack_device_encode(stream, source.data_ptr(), m, k,
                                              views[6].data_ptr(), scratch.data_ptr(),
                                              *(v.data_ptr() for v in views[:6])))
    return PackedWeight(views, m, k, max_common, max_rare, start_exp, arena)


# ---------------------------------------------------------------- forward
def _buffers_problem(buffers: list[Tensor], device: torch.device) -> str | None:
    if len(buffers) != 7 or any(
        t.device != device or t.dtype != torch.uint8 or not t.is_contiguous() for t in buffers
    ):
        return "All seven ZipServ byte buffers must be contiguous on the input GPU"
    return None


def _indexing_problem(m: int, n: int, k: int, split_k: int) -> str | None:
    if max(m * n * split_k, k * n, m * k) > INT32_MAX or (m // 64) * split_k > 65535:
        return "ZipServ output and Split-K workspace exceed native int32 indexing"
    return None


def _linear_problem(x: Tensor, buffers: list[Tensor], m: int, k: int, split_k: int) -> str | None:
    """First violated contract of a fused call, checked in the reference's
    order (runtime.py:213-237 of the reference module)."""
    if m <= 0 or k <= 0 or m % 64 or k % 64:
        return "ZipServ linear requires positive, 64-aligned weight dimensions"
    if x.dtype != torch.bfloat16 or x.ndim < 1 or x.shape[-1] != k:
        return "ZipServ linear requires BF16 activations with the matching input width"
    if split_k < 1 or (k // 64) % split_k:
        return "Split-K must divide the number of 64-column weight tiles"
    problem = _buffers_problem(buffers, x.device)
    if problem:
        return problem
    tokens = x.numel() // k
    return _indexing_problem(m, tokens, k, split_k) if tokens else None


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
    problem = _linear_problem(x, buffers, m, k, split_k)
    if problem:
        raise ValueError(problem)
    tokens = x.numel() // k
    shape = (*x.shape[:-1], m)
    if tokens == 0:
        return x.new_empty(shape)
    lib = _cuda_library()
    if fp32_partials:
        require_fp32_partials()
    entry = lib.zipserv_mm_fp32 if fp32_partials else lib.zipserv_mm
    with torch.cuda.device(x.device):
        flat = x.reshape(tokens, k).contiguous()
        out = x.new_empty((tokens, m))
        # The kernel reduces K ranges itself (FP32, fixed order), so the
        # reference's [split_k, n, m] workspace is never needed: split 1 with
        # no workspace is a valid call for every split the caller asked for.
        _check(entry(_stream(x.device), *(b.data_ptr() for b in buffers), max_common,
                     max_rare, start_exp, flat.data_ptr(), out.data_ptr(), m, tokens, k, None, 1))
    return out.view(shape)


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
    part, ctr = _U64(0), _U64(0)
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
    problem = _buffers_problem(list(packed.buffers), x.device)
    if problem:
        raise ValueError(problem)
    n = x.numel() // k
    flat = x.reshape(n, k).contiguous()
    if out is None:
        out = x.new_empty((n, m))
    if n:
        problem = _indexing_problem(m, n, k, 1)
        if problem:
            raise ValueError(problem)
        lib = _cuda_library()
        head = (_stream(x.device), *(b.data_ptr() for b in packed.buffers), packed.max_common,
                packed.max_rare, packed.start_exp, flat.data_ptr(), out.data_ptr(), m, n, k,
                k_parts)
        if workspace is None:
            _check(lib.zipserv_mm_kparts(*head))
        else:
            partials, counters = workspace
            if partials.device != x.device or counters.device != x.device:
                raise ValueError("workspace must be on the activations' device")
            _check(lib.zipserv_mm_ws(*head, partials.data_ptr(),
                                     partials.numel() * partials.element_size(),
                                     counters.data_ptr(),
                                     counters.numel() * counters.element_size()))
    return out.reshape(*x.shape[:-1], m)


def plan_kparts(m: int, n: int, k: int) -> int:
    """CTAs per 128-row block of the default schedule on the current GPU
    (at least 1; the persistent grid may also give a CTA several blocks)."""
    return int(_cuda_library().zipserv_mm_plan(m, n, k))


def set_reducer_wait(ns: int) -> int:
    """How long (ns) a split row block's first K part waits for the others
    before the last-arrival reduction takes over (identical results; 0 sends
    every split row block that way). Returns the previous value."""
    return int(_cuda_library().zipserv_mm_reducer_wait(int(ns)))


def device_flags(clear: bool = True) -> int:
    """Device-side failure flags (bit 0: a kernel wait gave up, that launch's
    output is undefined). Synchronises the current device."""
    flags = ctypes.c_uint(0)
    _check(_cuda_library().zipserv_device_flags(ctypes.byref(flags), int(clear)))
    return int(flags.value)


def check_device() -> None:
    """Synchronise and raise if any kernel wait gave up since the last check
    (call at a point where a sync is acceptable, e.g. after a step)."""
    flags = device_flags(clear=True)
    if flags:
        raise RuntimeError(f"ZipServ kernel wait gave up (device flags {flags:#x}); "
                           "outputs since the last check are undefined")


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
    problem = _buffers_problem(list(packed.buffers), device)
    if problem:
        raise ValueError(problem)
    lib = _cuda_library()
    with torch.cuda.device(device):
        if out is None:
            out = torch.empty((packed.m, packed.k), dtype=torch.bfloat16, device=device)
        _check(lib.zipserv_decode(_stream(device), *(b.data_ptr() for b in packed.buffers),
                                  packed.max_common, packed.max_rare, packed.start_exp,
                                  out.data_ptr(), packed.m, packed.k))
    return out


# ------------------------------------------------------- stored packed format
# File layout (little endian): 8-byte magic, u32 format version, u32 header
# bytes, i32 m, k, max_common, max_rare, start_exp, u32 reserved, u64
# lengths[7], 32-byte SHA-256 of the arena, then the arena bytes (the seven
# streams at ARENA_ALIGN offsets, exactly as PackedWeight.to lays them out).
PACKED_MAGIC = b"ZSTCATBE"
PACKED_VERSION = 1
_HEADER = struct.Struct("<8sII5iI7Q32s")


def expected_lengths(m: int, k: int, max_common: int, max_rare: int) -> dict[str, int]:
    """Stream lengths fixed by the shape: bitmaps (64 u64 per 64x64 tile),
    band offsets (8 i32 per tile) and tile offsets ((tiles + 1) i32 pairs).
    The payload streams depend on the data and are bounded by the capacities."""
    tiles = (m // 64) * (k // 64)
    return {"bitmap1": tiles * 512, "bitmap2": tiles * 512, "bitmap3": tiles * 512,
            "medium": tiles * 32, "global": (tiles + 1) * 8,
            "sm_max": tiles * (-(-max_common // 16) * 16),
            "rare_max": tiles * (-(-max_rare // 8) * 8) * 2}


def _layout_problem(m, k, max_common, max_rare, lengths) -> str | None:
    if m <= 0 or k <= 0 or m % 64 or k % 64 or m * k > 2**31 - 4097:
        return "stored weight has an invalid shape"
    if not (0 <= max_common <= 4096 and 0 <= max_rare <= 4096):
        return "stored weight has invalid payload capacities"
    want = expected_lengths(m, k, max_common, max_rare)
    names = dict(zip(BUFFER_NAMES, lengths, strict=True))
    for name in ("bitmap1", "bitmap2", "bitmap3", "medium", "global"):
        if names[name] != want[name]:
            return f"stored weight has a {name} stream of the wrong length"
    if names["sm"] > want["sm_max"] or names["rare"] > want["rare_max"]:
        return "stored weight has payload streams beyond their capacities"
    return None


def save_packed(packed: PackedWeight, path: str | os.PathLike) -> None:
    """Write a packed weight (any device) in the stored format."""
    host = packed.to("cpu")
    arena = host._own_arena()
    payload = arena.numpy().tobytes()
    header = _HEADER.pack(PACKED_MAGIC, PACKED_VERSION, _HEADER.size, host.m, host.k,
                          host.max_common, host.max_rare, host.start_exp, 0, *host.lengths,
                          hashlib.sha256(payload).digest())
    tmp = Path(str(path) + ".tmp")
    with open(tmp, "wb") as f:
        f.write(header)
        f.write(payload)
    os.replace(tmp, path)


def load_packed(path: str | os.PathLike, device: torch.device | str = "cpu") -> PackedWeight:
    """Read a stored packed weight, checking magic, version, stream lengths
    against the shape and the arena's SHA-256; then move it to `device`."""
    data = Path(path).read_bytes()
    if len(data) < _HEADER.size:
        raise ValueError("not a ZipServ packed weight (file too short)")
    magic, version, hbytes, m, k, mc, mr, se, _, *rest = _HEADER.unpack_from(data)
    lengths, digest = rest[:7], rest[7]
    if magic != PACKED_MAGIC:
        raise ValueError("not a ZipServ packed weight (bad magic)")
    if version != PACKED_VERSION or hbytes != _HEADER.size:
        raise ValueError(f"unsupported ZipServ packed format version {version}")
    problem = _layout_problem(m, k, mc, mr, lengths)
    if problem:
        raise ValueError(problem)
    payload = data[_HEADER.size:]
    if len(payload) != _arena_offsets(lengths)[1]:
        raise ValueError("stored weight is truncated or has trailing bytes")
    if hashlib.sha256(payload).digest() != digest:
        raise ValueError("stored weight fails its checksum")
    arena = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    packed = PackedWeight(_arena_views(arena, lengths), m, k, mc, mr, se, arena)
    return packed if torch.device(device).type == "cpu" else packed.to(device)
