"""Argument contracts of the C ABI, checked on the CPU.

The GPU entry points validate shapes, Split-K, packed maxima and pointers
before touching the device (csrc/L_API.cu:245-252, :344-351), so every
rejection below runs without a GPU. The expected verdicts come from the
oracle's restatement of csrc/CodecUtils.h:11-36 (oracle_valid_*), itself
exercised on the edge cases of tests/test_codec_utils.cpp:10-24.
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from zipserv_asplos26_b200 import runtime

ROOT = Path(__file__).resolve().parents[1]
INT_MAX = 2**31 - 1
INVALID_VALUE = 1  # cudaErrorInvalidValue


def test_oracle_contract_edge_cases(oracle_mod):
    lib = oracle_mod.lib()
    # tests/test_codec_utils.cpp:10-24
    assert lib.oracle_valid_matrix(64, 64)
    assert not lib.oracle_valid_matrix(0, 64) and not lib.oracle_valid_matrix(64, 0)
    assert not lib.oracle_valid_matrix(-64, 64) and not lib.oracle_valid_matrix(96, 64)
    assert lib.oracle_valid_matrix(32768, 65472)          # 2^31 - 2^21 elements
    assert not lib.oracle_valid_matrix(65536, 65536)
    assert lib.oracle_valid_gemm(64, 0, 64, 1)             # N = 0 is a valid no-op
    assert not lib.oracle_valid_gemm(64, -1, 64, 1)
    assert lib.oracle_valid_gemm(64, 8, 256, 4) and not lib.oracle_valid_gemm(64, 8, 256, 3)
    assert not lib.oracle_valid_gemm(64, 8, 256, 0)
    assert not lib.oracle_valid_gemm(64 * 65536, 1, 64, 1)  # grid.y limit (M/64)*split
    assert lib.oracle_valid_counts(4096, 0) and lib.oracle_valid_counts(0, 4096)
    assert lib.oracle_valid_counts(4048, 120)
    assert not lib.oracle_valid_counts(4095, 8)            # common not a multiple of 16
    assert not lib.oracle_valid_counts(16, 12)             # rare not a multiple of 8
    assert not lib.oracle_valid_counts(4112, 0) and not lib.oracle_valid_counts(16, 8)


GEMM_CASES = [
    # (m, n, k, split)
    (64, 1, 64, 1), (64, 0, 64, 1), (64, 8, 256, 4), (64, 8, 256, 3), (64, 8, 256, 0),
    (0, 8, 64, 1), (64, 8, 0, 1), (96, 8, 64, 1), (64, 8, 96, 1), (64, -1, 64, 1),
    (64 * 65536, 1, 64, 1), (4096, 1 << 20, 4096, 1), (65536, 32768, 64, 1),
    (4096, 1024, 4096, 64), (4096, 16, 4096, 16),
]


@pytest.mark.parametrize("m,n,k,split", GEMM_CASES)
def test_mm_shape_contract_matches_oracle(native_lib, oracle_mod, m, n, k, split):
    """Rejected shapes return cudaErrorInvalidValue before any device work;
    accepted shapes with N = 0 return success without a launch."""
    ok = bool(oracle_mod.lib().oracle_valid_gemm(m, n, k, split))
    args = [None] * 7 + [4048, 120, 115, None, None, m, n, k, None, split]
    fn = native_lib.zipserv_mm
    if not ok:
        assert fn(None, *args) == INVALID_VALUE
        assert native_lib.zipserv_mm_fp32(None, *args) == INVALID_VALUE
        assert b"invalid" in native_lib.zipserv_error()
    elif n == 0:
        assert fn(None, *args) == 0
    else:
        # Valid shape, null buffers: rejected as null pointers, still host-side.
        assert fn(None, *args) == INVALID_VALUE
        assert b"null" in native_lib.zipserv_error()


@pytest.mark.parametrize("counts", [(4096, 0), (0, 4096), (4095, 8), (16, 12), (4112, 0),
                                    (16, 8), (4048, 120)])
def test_mm_counts_contract(native_lib, oracle_mod, counts):
    ok = bool(oracle_mod.lib().oracle_valid_counts(*counts))
    r = native_lib.zipserv_mm(None, *[None] * 7, *counts, 115, None, None, 64, 0, 64, None, 1)
    assert r == (0 if ok else INVALID_VALUE)


def test_decode_contract(native_lib):
    dec = native_lib.zipserv_decode
    base = [None] * 7 + [4048, 120, 115, None]
    assert dec(None, *base, 64, 64) == INVALID_VALUE                 # null pointers
    assert b"null" in native_lib.zipserv_error()
    for m, k in ((0, 64), (64, 0), (96, 64), (64 * 65536, 64)):
        assert dec(None, *base, m, k) == INVALID_VALUE
        assert b"invalid" in native_lib.zipserv_error()
    assert dec(None, *[None] * 7, 4095, 8, 115, None, 64, 64) == INVALID_VALUE


def test_unaligned_pointers_rejected_before_launch(native_lib):
    """16-byte alignment is an extra precondition of the bulk/tensor copies."""
    buf = np.zeros(4096, dtype=np.uint8)
    p = buf.ctypes.data
    p16 = (p + 15) & ~15
    ptrs = [p16] * 7
    ok_args = ptrs + [4048, 120, 115, p16, p16, 64, 1, 64, None, 1]
    bad = list(ok_args)
    bad[2] = p16 + 8  # b1
    assert native_lib.zipserv_mm(None, *bad) == INVALID_VALUE
    assert b"aligned" in native_lib.zipserv_error()
    bad = list(ok_args)
    bad[11] = p16 + 4  # x
    assert native_lib.zipserv_mm(None, *bad) == INVALID_VALUE
    assert native_lib.zipserv_mm_kparts(None, *ptrs, 4048, 120, 115, p16, p16 + 2, 64, 1, 64,
                                        0) == INVALID_VALUE


def test_kparts_range(native_lib):
    args = [None] * 7 + [4048, 120, 115, None, None]
    for kparts in (-1, 17, 5):  # K = 256 has 4 tiles
        assert native_lib.zipserv_mm_kparts(None, *args, 64, 1, 256, kparts) == INVALID_VALUE
    assert native_lib.zipserv_mm_kparts(None, *args, 64, 0, 256, 4) == 0
    assert native_lib.zipserv_mm_plan(64, 1, 96) == -1


def _declared_c_symbols() -> list[str]:
    text = (ROOT / "include" / "zipserv_bridge.h").read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(zipserv_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(native_lib):
    names = _declared_c_symbols()
    assert {"zipserv_error", "zipserv_abi_version", "zipserv_free", "zipserv_compress",
            "zipserv_mm", "zipserv_mm_fp32", "zipserv_decode"} <= set(names)
    for name in names:
        assert hasattr(native_lib, name), name
    assert native_lib.zipserv_abi_version() == 2
    exported = subprocess.run(["nm", "-DC", "--defined-only", str(runtime.library_path())],
                              check=True, capture_output=True, text=True).stdout
    # include/L_API.h declares four C++ entry points (build/L_API.cuh:32-102).
    for sig in ("BF16TripleBitmap_MM_API(CUstream_st*, unsigned char const*, __nv_bfloat16 const*",
                "BF16TripleBitmap_MM_API_FP32(CUstream_st*, unsigned char const*",
                "BF16TripleBitmap_Decompress_API(CUstream_st*, unsigned char const*",
                "InitBF16MatrixTripleBitmap(__nv_bfloat16*, int, int, int, int, int, int, int, int, "
                "int const*"):
        assert sig in exported, sig


def test_l_api_header_declares_reference_entry_points():
    text = (ROOT / "include" / "L_API.h").read_text()
    for name in ("BF16TripleBitmap_MM_API", "BF16TripleBitmap_MM_API_FP32",
                 "BF16TripleBitmap_Decompress_API", "InitBF16MatrixTripleBitmap"):
        assert re.search(rf"\b{name}\s*\(", text), name


def test_fused_allreduce_sizes_and_argument_checks(native_lib):
    """zipserv_mm_allreduce_sizes: receive buffer = 2 parities x world x the
    [N tile x 128] values of every unit, one 64-bit word each (FP32 value and
    launch tag); the flag area is reserved (16 bytes). Invalid worlds and
    exchanges are refused before any GPU work."""
    rb, fb = ctypes.c_uint64(0), ctypes.c_uint64(0)
    assert native_lib.zipserv_mm_allreduce_sizes(4096, 16, 2, ctypes.byref(rb), ctypes.byref(fb)) == 0
    units = 4096 // 128
    assert rb.value == 2 * 2 * units * 16 * 128 * 8
    assert fb.value == 16
    assert native_lib.zipserv_mm_allreduce_sizes(4096, 16, 1, ctypes.byref(rb), ctypes.byref(fb)) == 1
    assert native_lib.zipserv_mm_allreduce_sizes(4096, 16, 9, ctypes.byref(rb), ctypes.byref(fb)) == 1
    bufs = [None] * 7
    for world, rank in ((1, 0), (9, 0), (2, 2), (2, -1)):
        assert native_lib.zipserv_mm_allreduce(None, *bufs, 4048, 120, 115, None, None, 4096, 16,
                                               4096, world, rank, None, None, None, 0, 0) == 1
        assert b"world" in native_lib.zipserv_error()
