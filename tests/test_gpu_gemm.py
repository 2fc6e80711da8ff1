"""Fused ZipGEMM parity through the C ABI (zipserv_mm / zipserv_mm_fp32 /
zipserv_mm_kparts) against the CPU oracle.

* Integer-valued operands (tests/test_cuda.cu:110-165): every FP32 sum is
  exact, so outputs must match the oracle bit for bit for every N tail, every
  K partition and both packing windows; 0x55 guard words after the output
  must survive.
* Real-valued weights ~N(0, 0.02) and activations ~N(0, 1): max relative
  error <= 1e-2 and mean relative error <= 1e-3 against the oracle's
  FP32-accumulated GEMM on the identical decoded weights.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import MAX_REL_TOL, MEAN_REL_TOL, bf16_tensor, make_packed, rel_errors, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu

N_VALUES = (1, 3, 7, 8, 9, 16, 17, 31, 32, 33, 48, 49, 64, 65, 80, 81, 96, 97, 112, 113, 127,
            128, 129, 193)
GUARD = 256


def call_mm(packed, x_dev, n, y_buf, *, kparts=None, split=1, workspace=None, fp32=False):
    lib = runtime._cuda_library()
    stream = torch.cuda.current_stream().cuda_stream
    args = [b.data_ptr() for b in packed.buffers]
    ws = workspace.data_ptr() if workspace is not None else None
    if kparts is not None:
        return lib.zipserv_mm_kparts(stream, *args, packed.max_common, packed.max_rare,
                                     packed.start_exp, x_dev.data_ptr(), y_buf.data_ptr(),
                                     packed.m, n, packed.k, kparts)
    fn = lib.zipserv_mm_fp32 if fp32 else lib.zipserv_mm
    return fn(stream, *args, packed.max_common, packed.max_rare, packed.start_exp,
              x_dev.data_ptr(), y_buf.data_ptr(), packed.m, n, packed.k, ws, split)


def guarded(n, m):
    return torch.full((n * m + GUARD,), 0x5555, dtype=torch.int16, device="cuda").view(torch.bfloat16)


@pytest.mark.parametrize("k", [64, 128, 512])
@pytest.mark.parametrize("window", [121, 100])
def test_integer_gemm_exact(native_lib, oracle_mod, k, window):
    m = 64
    rng = oracle_mod.MT19937(42 + k + window)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    p = oracle_mod.pack(w, window)  # 121: common+rare mix, 100: everything rare
    packed = make_packed(p, m, k).to("cuda")
    kt = k // 64
    for n in N_VALUES:
        x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
        expected, _ = oracle_mod.gemm(w, x)
        x_dev = bf16_tensor(x).cuda()
        for kparts in sorted({0, 1, 2, 4, 8, kt} & set(range(0, kt + 1))):
            y = guarded(n, m)
            assert call_mm(packed, x_dev, n, y, kparts=kparts) == 0
            torch.cuda.synchronize()
            got = words_of(y)
            assert np.array_equal(got[: n * m].reshape(n, m), expected), (n, kparts)
            assert np.all(got[n * m:] == 0x5555), (n, kparts)
        for split in (1, 2, 4, 8):
            if kt % split:
                continue
            y = guarded(n, m)
            ws = torch.full((split * n * m + GUARD,), 0x5555, dtype=torch.int16, device="cuda")
            assert call_mm(packed, x_dev, n, y, split=split, workspace=ws) == 0
            torch.cuda.synchronize()
            got = words_of(y)
            assert np.array_equal(got[: n * m].reshape(n, m), expected), (n, split)
            assert np.all(got[n * m:] == 0x5555)
            # The reduction happens in the kernel: the workspace is never written.
            assert torch.all(ws == 0x5555)
    assert runtime.device_flags() == 0


@pytest.mark.parametrize("m,k,n", [(128, 192, 9), (4096, 512, 129), (4096, 64, 147),
                                   (4032, 64, 160), (128, 64, 1), (192, 256, 300)])
def test_integer_gemm_fp32_api(native_lib, oracle_mod, m, k, n):
    """tests/test_cuda.cu:171-233 shapes: output exact, guards on both sides of
    the output and of the (untouched) FP32 workspace."""
    rng = oracle_mod.MT19937(7 + m + k + n)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    expected, _ = oracle_mod.gemm(w, x)
    split = max(s for s in (1, 2, 3, 4) if (k // 64) % s == 0)
    y = torch.full((n * m + 256,), 0x5555, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    ws = torch.full((split * n * m + 256,), 0x55555555, dtype=torch.int32, device="cuda")
    x_dev = bf16_tensor(x).cuda()
    y_view = y[128:]
    ws_view = ws[128:]
    assert call_mm(packed, x_dev, n, y_view, split=split, workspace=ws_view, fp32=True) == 0
    torch.cuda.synchronize()
    got = words_of(y)
    assert np.array_equal(got[128:128 + n * m].reshape(n, m), expected)
    assert np.all(got[:128] == 0x5555) and np.all(got[128 + n * m:] == 0x5555)
    assert torch.all(ws == 0x55555555)


def test_invalid_arguments(native_lib, oracle_mod):
    w = oracle_mod.integer_matrix(oracle_mod.MT19937(1), 64 * 128).reshape(64, 128)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    lib = runtime._cuda_library()
    stream = torch.cuda.current_stream().cuda_stream
    args = [b.data_ptr() for b in packed.buffers]
    meta = (packed.max_common, packed.max_rare, packed.start_exp)
    # tests/test_cuda.cu:161-165
    assert lib.zipserv_mm(stream, *args, *meta, None, None, 64, 1, 128, None, 1) == 1
    assert lib.zipserv_mm(stream, *args, *meta, None, None, 64, -1, 128, None, 1) == 1
    assert lib.zipserv_mm(stream, *args, *meta, None, None, 64, 1, 128, None, 0) == 1
    assert lib.zipserv_mm(stream, *args, *meta, None, None, 64, 1, 128, None, 3) == 1
    assert lib.zipserv_mm(stream, *args, *meta, None, None, 64, 0, 128, None, 1) == 0
    assert lib.zipserv_mm_fp32(stream, *args, *meta, None, None, 64, 0, 128, None, 2) == 0
    # Split-K > 1 still requires its workspace, as in the reference.
    x = torch.zeros(1, 128, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(1, 64, dtype=torch.bfloat16, device="cuda")
    assert lib.zipserv_mm(stream, *args, *meta, x.data_ptr(), y.data_ptr(), 64, 1, 128, None, 2) == 1
    assert b"null" in lib.zipserv_error()
    # Misaligned activations are rejected, not faulted on.
    xb = torch.zeros(2 * 128 + 8, dtype=torch.bfloat16, device="cuda")
    assert lib.zipserv_mm(stream, *args, *meta, xb.data_ptr() + 2, y.data_ptr(), 64, 1, 128,
                          None, 1) == 1
    # Bad packed maxima (valid_counts, csrc/CodecUtils.h:26-29).
    assert lib.zipserv_mm(stream, *args, 4095, 0, packed.start_exp, x.data_ptr(), y.data_ptr(),
                          64, 1, 128, None, 1) == 1


@pytest.mark.parametrize("m,k", [(256, 512), (4096, 4096), (6144, 4096)])
def test_real_valued_gemm_tolerance(native_lib, oracle_mod, m, k):
    w = oracle_mod.llama_weight(m, k, seed=0)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    g = torch.Generator().manual_seed(1)
    ns = (1, 8, 16, 33, 64, 128, 256) if m <= 256 else (1, 16, 128)
    for n in ns:
        x = torch.randn(n, k, generator=g).to(torch.bfloat16)
        expected, _ = oracle_mod.gemm(w, words_of(x), threads=8)
        y = runtime.linear(x.cuda(), packed)
        torch.cuda.synchronize()
        mx, mean = rel_errors(words_of(y), expected)
        assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (n, mx, mean)
    assert runtime.device_flags() == 0


def test_kparts_agree_and_are_deterministic(native_lib, oracle_mod):
    m, k, n = 512, 2048, 24
    w = oracle_mod.llama_weight(m, k, seed=5, outliers=0.02)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    x = torch.randn(n, k, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    expected, _ = oracle_mod.gemm(w, words_of(x), threads=8)
    for kparts in (1, 2, 3, 4, 5, 8, 12, 16):
        a = runtime.linear_kparts(x, packed, kparts)
        b = runtime.linear_kparts(x, packed, kparts)
        torch.cuda.synchronize()
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), kparts
        mx, mean = rel_errors(words_of(a), expected)
        assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (kparts, mx, mean)


def test_large_n_tiles(native_lib, oracle_mod):
    m, k, n = 128, 256, 600  # three N tiles, the last partial
    rng = oracle_mod.MT19937(9)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    expected, _ = oracle_mod.gemm(w, x)
    y = runtime.linear(bf16_tensor(x).cuda(), packed)
    torch.cuda.synchronize()
    assert np.array_equal(words_of(y), expected)


def test_cuda_graph_capture_and_streams(native_lib, oracle_mod):
    m, k, n = 256, 256, 9
    rng = oracle_mod.MT19937(3)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
    expected, _ = oracle_mod.gemm(w, x)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    x_dev = bf16_tensor(x).cuda()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        runtime.linear(x_dev, packed, split_k=2)  # warm-up outside capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            y = runtime.linear(x_dev, packed, split_k=2)
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(words_of(y), expected)


def scattered(packed: runtime.PackedWeight) -> runtime.PackedWeight:
    """The same streams at unequal distances (bitmap planes not equally
    spaced), so the kernels take their per-plane copy path."""
    sizes = [b.numel() for b in packed.buffers]
    offsets, total = [], 0
    for i, size in enumerate(sizes):
        offsets.append(total)
        total += (size + 255) // 256 * 256 + 256 * (i + 1)
    storage = torch.zeros(total, dtype=torch.uint8, device="cuda")
    views = []
    for b, off in zip(packed.buffers, offsets):
        v = storage[off:off + b.numel()]
        v.copy_(b)
        views.append(v)
    return runtime.PackedWeight(tuple(views), packed.m, packed.k, packed.max_common,
                                packed.max_rare, packed.start_exp)


@pytest.mark.parametrize("m,k", [(192, 640), (64, 64), (320, 2112)])
def test_unequally_spaced_bitmaps(native_lib, oracle_mod, m, k):
    rng = oracle_mod.MT19937(m + k)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    cpu = runtime.compress(bf16_tensor(w))
    packed = scattered(cpu)
    planes = [b.data_ptr() for b in packed.buffers[2:5]]
    assert planes[1] - planes[0] != planes[2] - planes[1]
    for n in (1, 17, 64):
        x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
        expected, _ = oracle_mod.gemm(w, x)
        x_dev = bf16_tensor(x).cuda()
        for kparts in sorted({1, min(3, k // 64)}):
            y = runtime.linear_kparts(x_dev, packed, kparts)
            torch.cuda.synchronize()
            assert np.array_equal(words_of(y), expected), (n, kparts)
    dense = runtime.decompress(packed)
    torch.cuda.synchronize()
    assert np.array_equal(words_of(dense), w)
    assert runtime.device_flags() == 0


@pytest.mark.parametrize("m,k,n,kparts", [(640, 1024, 40, 3), (256, 1024, 600, 5),
                                          (192, 4096, 16, 0), (64, 64, 1, 0),
                                          (4096, 1024, 8, 8), (4160, 1024, 24, 16)])
def test_split_rows_exact(native_lib, oracle_mod, m, k, n, kparts):
    """Uneven CTA ranges: CTAs whose first and last row blocks are both split,
    several N tiles, row blocks with one tile row; grids larger than the GPU
    (reduced by the last CTA to arrive instead of a waiting first part);
    integer operands, exact."""
    rng = oracle_mod.MT19937(m + k + n)
    w = oracle_mod.integer_matrix(rng, m * k).reshape(m, k)
    x = oracle_mod.integer_matrix(rng, n * k).reshape(n, k)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    expected, _ = oracle_mod.gemm(w, x)
    y = runtime.linear_kparts(bf16_tensor(x).cuda(), packed, kparts)
    torch.cuda.synchronize()
    assert np.array_equal(words_of(y), expected)
    assert runtime.device_flags() == 0


def test_caller_workspace(native_lib, oracle_mod):
    """zipserv_mm_ws: caller scratch gives the library path's exact words,
    one pair of buffers serves launches of different shapes in any order (the
    counters return to zero), and undersized scratch is rejected."""
    k = 2048
    shapes = [(512, 24, 0), (512, 24, 3), (256, 300, 5), (512, 24, 16), (1024, 7, 0)]
    sizes = [runtime.workspace_size(m, n, k, kp) for m, n, kp in shapes]
    assert all(p > 0 and c > 0 for p, c in sizes)  # every shape here splits row blocks
    partials = torch.full((max(p for p, _ in sizes),), 0x5A, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(max(c for _, c in sizes), dtype=torch.uint8, device="cuda")
    weights = {}
    for rep in range(2):
        for m, n, kp in (shapes if rep == 0 else shapes[::-1]):
            if m not in weights:
                w = oracle_mod.llama_weight(m, k, seed=7, outliers=0.02)
                weights[m] = runtime.compress(bf16_tensor(w)).to("cuda")
            packed = weights[m]
            x = torch.randn(n, k, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16).cuda()
            ref = runtime.linear_kparts(x, packed, kp)
            got = runtime.linear_kparts(x, packed, kp, workspace=(partials, counters))
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), (m, n, kp)
            assert int(counters.count_nonzero()) == 0
    p, c = sizes[0]
    with pytest.raises(RuntimeError):
        runtime.linear_kparts(x, weights[512], 0, workspace=(partials[: p - 16], counters))
    # One CTA per row block splits nothing and needs no scratch.
    assert runtime.workspace_size(256, 16, 256, 1) == (0, 0)
    assert runtime.device_flags() == 0
