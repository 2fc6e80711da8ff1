"""zipserv_mm_noalloc, the fused GEMM for callers that cannot allocate device
memory (bindings that only hold the buffers they are given, engines whose
memory is fully committed at start-up): its K-range scratch is a fixed array
in the library's device memory instead of a cudaMalloc'd buffer.

Called through the C ABI, it must give exactly the words zipserv_mm gives on
the same inputs (both run the same deterministic schedule and K-order
reduction), within the parity tolerance of the CPU oracle's FP32 GEMM,
including on consecutive calls, which reuse the array the previous call left
behind; shapes that need more scratch than the array holds are refused with a
clear error. This file is
collected last, so a run that stops at the first failure has run every
other test first."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import MAX_REL_TOL, MEAN_REL_TOL, bf16_tensor, rel_errors, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu

M = K = 4096  # an o-projection: every schedule splits row blocks over CTAs


@pytest.fixture(scope="module")
def lib(native_lib):
    lib = runtime._cuda_library()
    ptr, i32 = ctypes.c_void_p, ctypes.c_int
    lib.zipserv_mm_noalloc.argtypes = [ptr] * 8 + [i32] * 3 + [ptr] * 2 + [i32] * 4
    lib.zipserv_mm_noalloc.restype = i32
    return lib


@pytest.fixture(scope="module")
def weight(oracle_mod):
    return oracle_mod.llama_weight(M, K, seed=21)


@pytest.fixture(scope="module")
def packed(native_lib, weight):
    return runtime.compress(bf16_tensor(weight)).to("cuda")


def _args(packed):
    return [b.data_ptr() for b in packed.buffers]


def _noalloc(lib, packed, x, n):
    y = torch.empty(n, M, dtype=torch.bfloat16, device="cuda")
    rc = lib.zipserv_mm_noalloc(torch.cuda.current_stream().cuda_stream, *_args(packed),
                                packed.max_common, packed.max_rare, packed.start_exp,
                                x.data_ptr(), y.data_ptr(), M, n, K, 0)
    return rc, y


def _mm(lib, packed, x, n):
    y = torch.empty(n, M, dtype=torch.bfloat16, device="cuda")
    rc = lib.zipserv_mm(torch.cuda.current_stream().cuda_stream, *_args(packed),
                        packed.max_common, packed.max_rare, packed.start_exp, x.data_ptr(),
                        y.data_ptr(), M, n, K, None, 1)
    return rc, y


def test_matches_zipserv_mm_on_consecutive_calls(lib, packed, weight, oracle_mod):
    g = torch.Generator().manual_seed(7)
    for n in (16, 64):  # two calls in a row; the second reuses the first's scratch
        partial, counters = runtime.workspace_size(M, n, K)
        assert partial > 0 and counters > 0  # the fixed scratch is really used
        x = torch.randn(n, K, generator=g).to(torch.bfloat16)
        x_dev = x.cuda()
        rc, got = _noalloc(lib, packed, x_dev, n)
        assert rc == 0, lib.zipserv_error()
        rc, want = _mm(lib, packed, x_dev, n)
        assert rc == 0, lib.zipserv_error()
        torch.cuda.synchronize()
        assert runtime.device_flags() == 0
        assert np.array_equal(words_of(got), words_of(want)), n
        expected, _ = oracle_mod.gemm(weight, words_of(x), threads=8)
        mx, mean = rel_errors(words_of(got), expected)
        assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (n, mx, mean)


def test_refuses_shapes_beyond_the_fixed_scratch(lib, packed):
    n = 256  # a 256-token tile needs about 39 MB of partial tiles
    x = torch.zeros(n, K, dtype=torch.bfloat16, device="cuda")
    rc, _ = _noalloc(lib, packed, x, n)
    assert rc == 1  # cudaErrorInvalidValue
    assert b"fixed scratch" in lib.zipserv_error()
