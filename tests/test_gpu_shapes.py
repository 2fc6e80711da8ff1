"""Fused ZipGEMM parity at the benchmarked and configured shapes.

* The four Llama-3-8B linears at full size (the benchmark sweep), including
  gate_up 28672x4096 and down 4096x14336 whose K/64 = 224 gives the persistent
  schedule different segment boundaries, and 4096x4096 at N = 8 (the CPU-runnable configuration,
  the reference's `test_mm 4096 4096 8 1` shape).
* One row-parallel shard per tensor-parallel degree (o and down split on K
  at TP 2/4/8, the Llama-3-70B down shard K = 3584) and the 70B column shards.
* The C++ L_API entry points (build/L_API.cuh:32-74) called on the device
  through their mangled names.
* The reference's own Python runtime (integrations/vllm/zipserv_vllm/
  runtime.py) bound to this library through ZIPSERV_LIBRARY, as a vLLM
  deployment of the reference would run it (check_runtime.py:36-70).

Tolerance (the hot path's specification): max relative error <= 1e-2 and mean
relative error <= 1e-3 against an FP32-accumulated product of the identical,
bit-exactly decoded weight (tests/test_cuda.cu:125-131 restated as an FP32
torch matmul with TF32 off, which is what the CPU oracle computes).
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import MAX_REL_TOL, MEAN_REL_TOL, bf16_tensor, rel_errors, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _fp32_reference(w_dev: torch.Tensor, x_dev: torch.Tensor) -> np.ndarray:
    """bf16(x @ w^T) with FP32 products and sums (TF32 disabled)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y = (x_dev.float() @ w_dev.float().t()).to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return words_of(y)


def _weight(oracle_mod, m, k, seed):
    w = oracle_mod.llama_weight(m, k, seed=seed)
    return w, runtime.compress(bf16_tensor(w)).to("cuda")


def _check_linear(w, packed, ns, seed):
    w_dev = bf16_tensor(w).cuda()
    dense = runtime.decompress(packed)
    torch.cuda.synchronize()
    assert torch.equal(dense.view(torch.int16), w_dev.view(torch.int16)), "decode not bit-exact"
    g = torch.Generator().manual_seed(seed)
    for n in ns:
        x = torch.randn(n, packed.k, generator=g).to(torch.bfloat16).cuda()
        y = runtime.linear(x, packed)
        y2 = runtime.linear(x, packed)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), (n, "not deterministic")
        mx, mean = rel_errors(words_of(y), _fp32_reference(w_dev, x))
        assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (packed.m, packed.k, n, mx, mean)
    assert runtime.device_flags() == 0


@pytest.mark.parametrize("name,m,k", [("qkv", 6144, 4096), ("o", 4096, 4096),
                                      ("gate_up", 28672, 4096), ("down", 4096, 14336)])
def test_llama3_8b_linears_full_size(native_lib, oracle_mod, name, m, k):
    w, packed = _weight(oracle_mod, m, k, seed=1000 + len(name))
    _check_linear(w, packed, (1, 8, 16, 64, 128), seed=m + k)


def test_config0_shape_against_cpu_oracle(native_lib, oracle_mod):
    """4096 x 4096, N = 8, weights seed 0 and activations seed 1 (the
    CPU-runnable configuration), against the CPU oracle's own FP32 GEMM."""
    m = k = 4096
    w = oracle_mod.llama_weight(m, k, seed=0)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    x = torch.randn(8, k, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    expected, _ = oracle_mod.gemm(w, words_of(x), threads=os.cpu_count() or 1)
    y = runtime.linear(x.cuda(), packed)
    torch.cuda.synchronize()
    mx, mean = rel_errors(words_of(y), expected)
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)


@pytest.mark.parametrize("m,k", [
    (4096, 2048), (4096, 1024), (4096, 512),      # 8B o split on K at TP 2/4/8
    (4096, 7168), (4096, 3584), (4096, 1792),     # 8B down split on K at TP 2/4/8
    (8192, 3584), (8192, 1024),                   # 70B down / o at TP 8
    (1280, 8192), (7168, 8192),                   # 70B qkv / gate_up column shards at TP 8
])
def test_tensor_parallel_shards(native_lib, oracle_mod, m, k):
    w, packed = _weight(oracle_mod, m, k, seed=m ^ k)
    _check_linear(w, packed, (1, 16, 64, 256) if m * k <= 2**25 else (1, 16), seed=m + 3 * k)


# --- the C++ entry points of include/L_API.h, on the device -----------------

_MANGLED = {
    "mm": "_Z23BF16TripleBitmap_MM_APIP11CUstream_stPKhPK13__nv_bfloat16PKmS7_S7_PKiS9_iihS5_PS3_iiiSA_i",
    "mm_fp32": "_Z28BF16TripleBitmap_MM_API_FP32P11CUstream_stPKhPK13__nv_bfloat16PKmS7_S7_PKiS9_iihS5_PS3_iiiPfi",
    "decompress": "_Z31BF16TripleBitmap_Decompress_APIP11CUstream_stPKhPK13__nv_bfloat16PKmS7_S7_PKiS9_iihPS3_ii",
}


def _lapi(lib, which):
    fn = getattr(lib, _MANGLED[which])
    p, i = ctypes.c_void_p, ctypes.c_int
    if which == "decompress":
        fn.argtypes = [p] * 8 + [i, i, ctypes.c_uint8, p, i, i]
    else:
        fn.argtypes = [p] * 8 + [i, i, ctypes.c_uint8, p, p, i, i, i, p, i]
    fn.restype = i
    return fn


def test_lapi_cpp_entry_points_on_device(native_lib, oracle_mod):
    m, k = 512, 1024
    w = oracle_mod.llama_weight(m, k, seed=11, outliers=0.02)
    packed = runtime.compress(bf16_tensor(w)).to("cuda")
    lib = runtime._cuda_library()
    stream = torch.cuda.current_stream().cuda_stream
    bufs = [b.data_ptr() for b in packed.buffers]
    meta = (packed.max_common, packed.max_rare, packed.start_exp)
    out = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
    assert _lapi(lib, "decompress")(stream, *bufs, *meta, out.data_ptr(), m, k) == 0
    torch.cuda.synchronize()
    assert np.array_equal(words_of(out), w)
    w_dev = bf16_tensor(w).cuda()
    g = torch.Generator().manual_seed(3)
    for n in (1, 8, 33, 128):
        x = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
        ref = _fp32_reference(w_dev, x)
        for split in (1, 2, 4, 8):
            for which, dtype in (("mm", torch.bfloat16), ("mm_fp32", torch.float32)):
                y = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")
                ws = torch.zeros(split * n * m, dtype=dtype, device="cuda")
                rc = _lapi(lib, which)(stream, *bufs, *meta, x.data_ptr(), y.data_ptr(), m, n, k,
                                       ws.data_ptr(), split)
                assert rc == 0, lib.zipserv_error()
                torch.cuda.synchronize()
                mx, mean = rel_errors(words_of(y), ref)
                assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (which, n, split, mx, mean)
    # Contract violations return cudaErrorInvalidValue without a launch.
    y = torch.empty(1, m, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(1, k, dtype=torch.bfloat16, device="cuda")
    assert _lapi(lib, "mm")(stream, *bufs, *meta, x.data_ptr(), y.data_ptr(), m, 1, k, None, 2) == 1
    assert _lapi(lib, "mm")(stream, *bufs, *meta, x.data_ptr(), y.data_ptr(), m, 1, k, None, 3) == 1
    assert runtime.device_flags() == 0


# --- the reference's own runtime.py bound to this library --------------------

_REFERENCE_SCRIPT = r"""
import json, sys
import torch
sys.path.insert(0, sys.argv[1])                 # the repository (oracle: test checker only)
sys.path.append(sys.argv[2])                    # baseline/_ref (installed reference package)
from zipserv_vllm import runtime as ref_rt
from oracle import oracle
import numpy as np

def words(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

report = {"cases": []}
w = oracle.llama_weight(256, 1024, seed=5, outliers=0.01)
weight = torch.from_numpy(w.view(np.int16)).view(torch.bfloat16)
packed = ref_rt.compress(weight).to("cuda")
report["decode_exact"] = bool(np.array_equal(words(ref_rt.decompress(packed)), w))
g = torch.Generator().manual_seed(9)
for n in (1, 8, 17, 64, 128):
    x = torch.randn(n, 1024, generator=g).to(torch.bfloat16)
    expected, _ = oracle.gemm(w, words(x))
    e = (expected.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    for split_k in (1, 2, 4, 8):
        for partial in ("bf16", "fp32"):
            y = ref_rt.linear(x.cuda(), packed, split_k=split_k, partial_dtype=partial)
            a = (words(y).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
            d = np.abs(a - e)
            report["cases"].append({"n": n, "split_k": split_k, "partial": partial,
                                    "max_rel": float(d.max() / max(np.abs(e).max(), 1e-30)),
                                    "mean_rel": float(d.mean() / max(np.abs(e).mean(), 1e-30))})
# A graph capture of a shape the library has not launched yet (the reference
# runtime passes its own split_k workspace).
x = torch.randn(5, 1024, generator=g).to(torch.bfloat16).cuda()
stream = torch.cuda.Stream()
with torch.cuda.stream(stream):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        y = ref_rt.linear(x, packed, split_k=4)
graph.replay()
torch.cuda.synchronize()
expected, _ = oracle.gemm(w, words(x))
report["captured_exact_shape"] = list(y.shape)
e = (expected.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
a = (words(y).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
report["captured_max_rel"] = float(np.abs(a - e).max() / np.abs(e).max())
print(json.dumps(report))
"""


def test_reference_runtime_through_zipserv_library(native_lib):
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "zipserv_vllm" / "runtime.py").is_file():
        pytest.skip("reference package not installed in baseline/_ref")
    env = dict(os.environ, ZIPSERV_LIBRARY=str(runtime.library_path()))
    # A separate process: the reference registers the same torch custom op
    # name (zipserv_vllm::linear) as this package.
    proc = subprocess.run([sys.executable, "-c", _REFERENCE_SCRIPT, str(ROOT), str(ref)],
                          capture_output=True, text=True, env=env, timeout=600)
    assert proc.returncode == 0, proc.stderr[-4000:]
    report = json.loads(proc.stdout.strip().splitlines()[-1])
    assert report["decode_exact"]
    assert len(report["cases"]) == 5 * 4 * 2
    for case in report["cases"]:
        assert case["max_rel"] <= MAX_REL_TOL and case["mean_rel"] <= MEAN_REL_TOL, case
    assert report["captured_exact_shape"] == [5, 256]
    assert report["captured_max_rel"] <= MAX_REL_TOL
