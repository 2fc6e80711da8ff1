"""Python runtime contracts on the CPU (reference tests/test_runtime.py:18-88
and tests/test_host_runtime.py:22-238): input validation before the library
loads, a missing library, storage accounting, the arena that holds a packed
weight, fault injection around the native allocation (freed exactly once),
the stored packed format, the fake-tensor shape contract of the custom op,
and decode budgets.
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


def test_compress_returns_the_native_output_before_it_returns(native_lib, oracle_mod,
                                                              monkeypatch):
    """The encoder's native buffers are copied into the arena and freed at
    once: the packed weight owns plain tensor memory (no finalizer ties it to
    native allocations)."""
    released = []
    original = runtime._release
    monkeypatch.setattr(runtime, "_release",
                        lambda lib, d: (released.append(tuple(d.lengths)), original(lib, d)))
    w = _weights(192, 256, seed=3)
    packed = runtime.compress(w)
    assert len(released) == 1
    gc.collect()
    bufs = [b.numpy() for b in packed.buffers]
    restored = oracle_mod.decode(bufs, packed.m, packed.k, packed.start_exp)
    assert np.array_equal(restored, w.view(torch.int16).numpy().view(np.uint16))


def test_copy_failure_frees_the_native_output_once(native_lib, monkeypatch):
    """A failure while copying the encoder's output (here: the arena
    allocation) still returns the native allocation, exactly once
    (the reference's tests/test_host_runtime.py:198-230 asks the same of its
    zero-copy wrapping)."""
    released = []
    original = runtime._release
    monkeypatch.setattr(runtime, "_release",
                        lambda lib, d: (released.append(1), original(lib, d)))

    def failing_arena(*_a, **_k):
        raise MemoryError("simulated arena allocation failure")

    monkeypatch.setattr(runtime, "_new_arena", failing_arena)
    with pytest.raises(MemoryError):
        runtime.compress(_weights())
    assert released == [1]


def test_arena_layout(native_lib):
    """Buffers are views of one arena at 256-byte aligned offsets, so the
    three equally sized bitmap planes are equally spaced; moving to the same
    device keeps the arena, and buffers made elsewhere are gathered."""
    packed = runtime.compress(_weights(128, 256, seed=9))
    base = packed.arena.data_ptr()
    offsets = [b.data_ptr() - base for b in packed.buffers]
    assert all(o % runtime.ARENA_ALIGN == 0 for o in offsets)
    assert offsets[3] - offsets[2] == offsets[4] - offsets[3]
    assert packed.to("cpu").arena is packed.arena
    loose = runtime.PackedWeight(tuple(b.clone() for b in packed.buffers), packed.m, packed.k,
                                 packed.max_common, packed.max_rare, packed.start_exp)
    gathered = loose.to("cpu")
    assert gathered.arena is not None and gathered.arena is not packed.arena
    assert all(torch.equal(a, b) for a, b in zip(gathered.buffers, packed.buffers))


def test_stored_format_round_trip_and_guards(native_lib, tmp_path):
    packed = runtime.compress(_weights(128, 256, seed=11))
    path = tmp_path / "w.zstb"
    runtime.save_packed(packed, path)
    back = runtime.load_packed(path)
    assert (back.m, back.k, back.max_common, back.max_rare, back.start_exp) == (
        packed.m, packed.k, packed.max_common, packed.max_rare, packed.start_exp)
    assert all(torch.equal(a, b) for a, b in zip(back.buffers, packed.buffers))
    data = path.read_bytes()
    hdr = runtime._HEADER.size

    def rejected(blob, match):
        bad = tmp_path / "bad.zstb"
        bad.write_bytes(blob)
        with pytest.raises(ValueError, match=match):
            runtime.load_packed(bad)

    rejected(b"XXXXXXXX" + data[8:], "magic")
    rejected(data[:8] + (2).to_bytes(4, "little") + data[12:], "version")
    rejected(data[:hdr + 5] + bytes([data[hdr + 5] ^ 1]) + data[hdr + 6:], "checksum")
    rejected(data[:-256], "truncated")
    rejected(data[:10], "too short")
    # A bitmap stream whose length does not match the shape.
    fields = list(runtime._HEADER.unpack_from(data))
    fields[9 + 2] += 8  # lengths start at field 9; bitmap1 is the third
    rejected(runtime._HEADER.pack(*fields) + data[hdr:], "bitmap1")


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
