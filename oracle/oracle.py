"""TEST INFRASTRUCTURE ONLY: Python access to the C oracle (oracle/oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline / reference
arm may import this module, and only as the checker. The product package never
imports it.

Besides ctypes wrappers this module restates the input generators of the
reference's own tests (tests/test_host_packer.cpp:69-111,
tests/test_cuda.cu:96-121, tests/test_codec_utils.cpp:27-45) so the same seeded
cases can be rebuilt here and on the GPU box.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)


class _Packed(ctypes.Structure):
    _fields_ = [
        ("sm", _u8p), ("rare", _u16p), ("b1", _u64p), ("b2", _u64p), ("b3", _u64p),
        ("small", _i32p), ("medium", _i32p), ("global_", _i32p),
        ("tiles", ctypes.c_int32), ("base", ctypes.c_int32),
        ("max_common", ctypes.c_int32), ("max_rare", ctypes.c_int32),
        ("lengths", ctypes.c_uint64 * 8),
    ]


class _MT(ctypes.Structure):
    _fields_ = [("state", ctypes.c_uint32 * 624), ("index", ctypes.c_int)]


_LIB = None


def build() -> Path:
    """Compile the C oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.is_file():
            build()
        l = ctypes.CDLL(str(LIB_PATH))
        l.oracle_pack.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.POINTER(_Packed)]
        l.oracle_free.argtypes = [ctypes.POINTER(_Packed)]
        l.oracle_decode.argtypes = [_u8p, _u16p, _u64p, _u64p, _u64p, _i32p, _i32p,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p]
        l.oracle_decode_mt.argtypes = l.oracle_decode.argtypes + [ctypes.c_int]
        l.oracle_gemm.argtypes = [_u16p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  _u16p, _f32p, ctypes.c_int]
        l.oracle_gemm.restype = None
        l.oracle_gemm_split.argtypes = [_u16p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, _f32p, _u16p]
        l.oracle_gemm_split.restype = None
        l.oracle_best_window.argtypes = [_u64p, ctypes.c_int]
        l.oracle_exponent_bits.argtypes = [ctypes.c_uint8, ctypes.c_uint8]
        l.oracle_exponent_bits.restype = ctypes.c_uint16
        l.oracle_valid_gemm.argtypes = [ctypes.c_int] * 4
        l.oracle_valid_matrix.argtypes = [ctypes.c_int] * 2
        l.oracle_valid_counts.argtypes = [ctypes.c_int] * 2
        l.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        l.oracle_f32_to_bf16.restype = ctypes.c_uint16
        l.oracle_mt_seed.argtypes = [ctypes.POINTER(_MT), ctypes.c_uint32]
        l.oracle_mt_fill.argtypes = [ctypes.POINTER(_MT), _u32p, ctypes.c_size_t]
        _LIB = l
    return _LIB


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctype)


@dataclass
class OraclePacked:
    """Encoder output in the reference's buffer order (csrc/HostPacker.h:83-88)."""

    sm: np.ndarray
    rare: np.ndarray
    b1: np.ndarray
    b2: np.ndarray
    b3: np.ndarray
    small: np.ndarray | None
    medium: np.ndarray
    global_: np.ndarray
    tiles: int
    base: int
    max_common: int
    max_rare: int

    @property
    def start_exp(self) -> int:
        # integrations/vllm/native/host_bridge.cpp:33
        return (self.base - 1) & 255

    def abi_buffers(self) -> list[np.ndarray]:
        """The seven byte buffers in C-ABI order (small offsets dropped)."""
        return [b.view(np.uint8) for b in (self.sm, self.rare, self.b1, self.b2, self.b3,
                                          self.medium, self.global_)]

    def all_buffers(self) -> list[np.ndarray | None]:
        return [self.sm, self.rare, self.b1, self.b2, self.b3, self.small, self.medium,
                self.global_]


def pack(words: np.ndarray, base: int = -1, include_small: bool = False) -> OraclePacked:
    words = np.ascontiguousarray(words, dtype=np.uint16)
    m, k = words.shape
    out = _Packed()
    if lib().oracle_pack(_ptr(words, _u16p), m, k, base, int(include_small), ctypes.byref(out)):
        raise ValueError("oracle_pack rejected its arguments")
    try:
        t = out.tiles

        def take(ptr, count, dtype):
            if count == 0:
                return np.zeros(0, dtype=dtype)
            return np.ctypeslib.as_array(ptr, shape=(count,)).copy().astype(dtype, copy=False)

        g = take(out.global_, 2 * (t + 1), np.int32)
        return OraclePacked(
            sm=take(out.sm, int(g[2 * t]), np.uint8),
            rare=take(out.rare, int(g[2 * t + 1]), np.uint16),
            b1=take(out.b1, 64 * t, np.uint64),
            b2=take(out.b2, 64 * t, np.uint64),
            b3=take(out.b3, 64 * t, np.uint64),
            small=take(out.small, 128 * t, np.int32) if out.small else None,
            medium=take(out.medium, 8 * t, np.int32),
            global_=g, tiles=t, base=out.base,
            max_common=out.max_common, max_rare=out.max_rare)
    finally:
        lib().oracle_free(ctypes.byref(out))


def decode(buffers, m: int, k: int, start_exp: int, threads: int = 1) -> np.ndarray:
    """Bit-exact CPU decode of the seven ABI buffers; raises on inconsistency."""
    sm, rare, b1, b2, b3, medium, glob = (np.ascontiguousarray(b).view(np.uint8) for b in buffers)
    out = np.empty((m, k), dtype=np.uint16)
    sm = sm if sm.size else np.zeros(16, np.uint8)
    rare = rare if rare.size else np.zeros(16, np.uint8)
    status = lib().oracle_decode_mt(
        _ptr(sm, _u8p), _ptr(rare.view(np.uint16), _u16p), _ptr(b1.view(np.uint64), _u64p),
        _ptr(b2.view(np.uint64), _u64p), _ptr(b3.view(np.uint64), _u64p),
        _ptr(medium.view(np.int32), _i32p), _ptr(glob.view(np.int32), _i32p),
        m, k, start_exp, _ptr(out, _u16p), threads)
    if status:
        raise ValueError(f"packed buffers are inconsistent (oracle code {status})")
    return out


def gemm(w: np.ndarray, x: np.ndarray, threads: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """y[n, m] = bf16(sum_k w[m,k] x[n,k]) with FP32 sums in ascending k."""
    w = np.ascontiguousarray(w, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = w.shape
    n = x.shape[0]
    y = np.empty((n, m), dtype=np.uint16)
    yf = np.empty((n, m), dtype=np.float32)
    lib().oracle_gemm(_ptr(w, _u16p), _ptr(x, _u16p), m, n, k, _ptr(y, _u16p),
                      _ptr(yf, _f32p), threads)
    return y, yf


def gemm_split(w: np.ndarray, x: np.ndarray, split: int) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = w.shape
    n = x.shape[0]
    partials = np.empty((split, n, m), dtype=np.float32)
    y = np.empty((n, m), dtype=np.uint16)
    lib().oracle_gemm_split(_ptr(w, _u16p), _ptr(x, _u16p), m, n, k, split,
                            _ptr(partials, _f32p), _ptr(y, _u16p))
    return partials, y


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """Vectorised round-to-nearest-even, same rule as oracle_f32_to_bf16."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class MT19937:
    """std::mt19937 stream (restated in oracle.c)."""

    def __init__(self, seed: int):
        self._mt = _MT()
        lib().oracle_mt_seed(ctypes.byref(self._mt), seed)

    def take(self, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.uint32)
        if count:
            lib().oracle_mt_fill(ctypes.byref(self._mt), _ptr(out, _u32p), count)
        return out

    def __call__(self) -> int:
        return int(self.take(1)[0])


def digest(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


# --- Reference test case generators -----------------------------------------

def host_packer_cases():
    """Yield (name, words, m, k, base, include_small) in the order and with the
    random stream of tests/test_host_packer.cpp:69-111 (std::mt19937(42))."""
    rng = MT19937(42)
    all_words = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(256, 256)
    for base in (-1, 0, 120, 249):
        yield f"all_words_base{base}", all_words, 256, 256, base, True
    for base in range(250):
        r = rng.take(4096)
        e = np.where(r % 5 != 0, base + (r % 7).astype(np.int64), (r % 256).astype(np.int64))
        words = ((r & 0x807F) | (e.astype(np.uint32) << 7)).astype(np.uint16)
        yield f"window_{base}", words.reshape(64, 64), 64, 64, base, True
    for word in (0, 0x8000, 0x7F80, 0xFFFF):
        words = np.full((128, 128), word, dtype=np.uint16)
        for base in (-1, 0, 120, 249):
            yield f"const_{word:04x}_base{base}", words, 128, 128, base, True
    for count in (0, 1, 7, 8, 15, 16, 17, 4080, 4081, 4088, 4095, 4096):
        words = np.full(4096, 30 << 7, dtype=np.uint16)
        words[:count] = 120 << 7
        yield f"padding_{count}", words.reshape(64, 64), 64, 64, 120, True
    for m, k in ((64, 192), (128, 320), (320, 128), (1024, 1024)):
        words = rng.take(m * k).astype(np.uint16).reshape(m, k)
        for small in (False, True):
            yield f"random_{m}x{k}_small{int(small)}", words, m, k, -1, small
    mixed = np.empty((256, 256), dtype=np.uint16)
    for row in range(256):
        for col in range(256):
            tile = (row // 64) * 4 + col // 64
            if tile % 3 == 0:
                mixed[row, col] = 120 << 7
            elif tile % 3 == 1:
                mixed[row, col] = 40 << 7
            else:
                mixed[row, col] = rng() & 0xFFFF
    for small in (False, True):
        yield f"mixed_tiles_small{int(small)}", mixed, 256, 256, 120, small


def decode_modes():
    """tests/test_cuda.cu:96-107: all words, 9-bit patterns, NaN/Inf band, zeros."""
    i = np.arange(65536, dtype=np.uint32)
    modes = [
        i,
        (i & 255) | ((i & 256) << 7),
        0x7F80 | (i & 127) | ((i & 128) << 8),
        np.zeros_like(i),
    ]
    return [m.astype(np.uint16).reshape(256, 256) for m in modes]


def integer_matrix(rng: MT19937, count: int) -> np.ndarray:
    """Values in {-1, 0, 1} as BF16 bits: float(int(rng() % 3) - 1)
    (tests/test_cuda.cu:114,121)."""
    v = (rng.take(count) % 3).astype(np.int64) - 1
    table = np.array([0xBF80, 0x0000, 0x3F80], dtype=np.uint16)  # -1, 0, +1
    return table[v + 1]


def llama_weight(m: int, k: int, seed: int = 0, outliers: float = 0.0):
    """N(0, 0.02) BF16 weights as torch draws them on CPU (seeded Generator);
    with `outliers` > 0 that fraction is redrawn from N(0, 1) at seeded
    uniform positions (the exception-stress configuration)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(m, k, generator=g) * 0.02
    if outliers > 0:
        mask = torch.rand(m, k, generator=g) < outliers
        w = torch.where(mask, torch.randn(m, k, generator=g), w)
    return w.to(torch.bfloat16).view(torch.uint16).numpy()


def ensure_built() -> None:
    if not LIB_PATH.is_file() or os.path.getmtime(LIB_PATH) < os.path.getmtime(HERE / "oracle.c"):
        build()
