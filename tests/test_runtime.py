"""Python runtime contracts on the CPU (reference tests/test_runtime.py:18-88
and tests/test_host_runtime.py:22-238): input validation before the library
loads, a missing library, storage accounting, zero-copy buffer sharing and
ownership, fault injection around the native allocation (freed exactly
once), the fake-tensor shape contract of the custom op, and decode budgets.
"""
from __future__ import annotations

import ctypes
import gc
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from zipserv_asplos26_b200 import runtime

GOLDEN = Path(__file__).resolve().parent / "golden"


def _weights(m=128, k=192, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)


def test_compress_validates_before_loading_the_library(monkeypatch):
    def boom():
        raise AssertionError("library loaded before validation")

    monkeypatch.setattr(runtime, "_library", boom)
    bad = [
        torch.zeros(64, 64, dtype=torch.float32),
        torch.zeros(64, dtype=torch.bfloat16),
        torch.zeros(64, 64, 1, dtype=torch.bfloat16),
        torch.zeros(96, 64, dtype=torch.bfloat16),
        torch.zeros(64, 0, dtype=torch.bfloat16),
        torch.zeros(0, 64, dtype=torch.bfloat16),
    ]
    if torch.device("meta"):
        bad.append(torch.zeros(64, 64, dtype=torch.bfloat16, device="meta"))
    for tensor in bad:
        with pytest.raises(ValueError):
            runtime.compress(tensor)


def test_missing_library_is_reported(monkeypatch, tmp_path):
    monkeypatch.setenv("ZIPSERV_LIBRARY", str(tmp_path / "missing.so"))
    runtime._library.cache_clear()
    try:
        with pytest.raises(RuntimeError, match="does not exist"):
            runtime.compress(_weights())
    finally:
        monkeypatch.delenv("ZIPSERV_LIBRARY")
        runtime._library.cache_clear()


def test_storage_accounting_matches_reference_bridge(native_lib, oracle_mod):
    want = json.loads((GOLDEN / "reference_bridge.json").read_text())["o_proj_small_256x512"]
    w = oracle_mod.llama_weight(want["m"], want["k"], want["seed"])
    packed = runtime.compress(torch.from_numpy(w.view(np.int16)).view(torch.bfloat16))
    assert packed.storage_bytes == want["storage_bytes"] == sum(want["lengths"])
    assert [b.numel() for b in packed.buffers] == want["lengths"]
    assert (packed.m, packed.k, packed.max_common, packed.max_rare, packed.start_exp) == (
        want["m"], want["k"], want["max_common"], want["max_rare"], want["start_exp"])
    assert runtime.BUFFER_NAMES == ("sm", "rare", "bitmap1", "bitmap2", "bitmap3", "medium",
                                    "global")


def test_round_trip_and_to_cpu(native_lib, oracle_mod):
    w = _weights(192, 256, seed=5)
    packed = runtime.compress(w)
    moved = packed.to("cpu")
    assert all(torch.equal(a, b) for a, b in zip(packed.buffers, moved.buffers))
    bufs = [b.numpy() for b in moved.buffers]
    restored = oracle_mod.decode(bufs, packed.m, packed.k, packed.start_exp)
    assert np.array_equal(restored, w.view(torch.int16).numpy().view(np.uint16))


def test_buffers_share_native_memory_until_the_last_view(native_lib, monkeypatch):
    freed = []
    original = runtime._free_packed

    def counting_free(lib, native):
        freed.append(tuple(native.buffers))
        original(lib, native)

    monkeypatch.setattr(runtime, "_free_packed", counting_free)
    packed = runtime.compress(_weights())
    keep = packed.buffers[2]
    snapshot = keep.clone()
    del packed
    gc.collect()
    assert freed == []                     # one live view keeps the allocation
    assert torch.equal(keep, snapshot)
    del keep
    gc.collect()
    assert len(freed) == 1                 # released exactly once


def test_frombuffer_failure_frees_native_memory_once(native_lib, monkeypatch):
    """tests/test_host_runtime.py:198-230: a failure while wrapping buffers
    must release the native allocation exactly once."""
    freed = []
    original_free = runtime._free_packed
    monkeypatch.setattr(runtime, "_free_packed",
                        lambda lib, native: (freed.append(1), original_free(lib, native)))
    calls = {"n": 0}
    original = torch.frombuffer

    def flaky(*args, **kwargs):
        calls["n"] += 1
        if calls["n"] == 3:
            raise MemoryError("simulated frombuffer failure")
        return original(*args, **kwargs)

    monkeypatch.setattr(torch, "frombuffer", flaky)
    with pytest.raises(MemoryError):
        runtime.compress(_weights())
    gc.collect()
    assert len(freed) == 1


def test_owner_allocation_failure_frees_native_memory(native_lib, monkeypatch):
    calls = []
    lib = runtime._library()
    original = lib.zipserv_free

    class FailingOwner:
        def __init__(self, *_):
            raise MemoryError("simulated owner allocation failure")

    monkeypatch.setattr(runtime, "_NativeBufferOwner", FailingOwner)
    monkeypatch.setattr(lib, "zipserv_free", lambda p: (calls.append(1), original(p)))
    with pytest.raises(MemoryError):
        runtime.compress(_weights())
    assert len(calls) == 1


def test_native_validation_failure_raises_with_message(native_lib, monkeypatch):
    lib = runtime._library()
    monkeypatch.setattr(lib, "zipserv_compress", lambda *a: -1)
    with pytest.raises(RuntimeError, match="ZipServ native call failed"):
        runtime.compress(_weights())


def test_fake_tensor_shape_contract():
    """The custom op's fake implementation gives (*x.shape[:-1], m) without
    touching the library (tests/test_runtime.py:55-73)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(3, 5, 256, dtype=torch.bfloat16, device="cuda")
        buffers = [torch.empty(16, dtype=torch.uint8, device="cuda") for _ in range(7)]
        y = torch.ops.zipserv_vllm.linear(x, buffers, 128, 256, 4048, 120, 115, 1, False)
        assert tuple(y.shape) == (3, 5, 128) and y.dtype == torch.bfloat16
        empty = torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")
        assert tuple(torch.ops.zipserv_vllm.linear(empty, buffers, 64, 256, 0, 4096, 0, 2,
                                                   True).shape) == (0, 64)


def test_linear_argument_checks_on_cpu(native_lib):
    packed = runtime.compress(_weights(128, 256))
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="partial_dtype"):
        runtime.linear(x, packed, partial_dtype="fp16")
    # The custom op has a CUDA kernel only (device_types="cuda"), as in the
    # reference: CPU activations fail at dispatch instead of running elsewhere.
    with pytest.raises(NotImplementedError):
        runtime.linear(x, packed)
    with pytest.raises(ValueError, match="matching input width"):
        runtime.linear_kparts(torch.zeros(2, 128, dtype=torch.bfloat16), packed, 0)
    with pytest.raises(ValueError, match="CUDA"):
        runtime.linear_kparts(x, packed, 0)


def test_decompress_budget_and_device_checks(native_lib):
    packed = runtime.compress(_weights(128, 256))
    with pytest.raises(ValueError, match="budget"):
        runtime.decompress(packed, max_bytes=128 * 256 * 2 - 1)
    with pytest.raises(ValueError, match="nonnegative"):
        runtime.decompress(packed, max_bytes=-1)
    with pytest.raises(ValueError, match="CUDA"):
        runtime.decompress(packed, max_bytes=128 * 256 * 2)


def test_old_abi_library_is_rejected(monkeypatch):
    class Old:
        def __init__(self, *_):
            self.zipserv_abi_version = lambda: 1

    monkeypatch.setattr(ctypes, "CDLL", Old)
    runtime._library.cache_clear()
    try:
        with pytest.raises(RuntimeError, match="ABI"):
            runtime._library()
    finally:
        monkeypatch.undo()
        runtime._library.cache_clear()
