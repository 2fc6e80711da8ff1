"""Pins the CPU oracle (oracle/oracle.c) to the reference's own outputs.

The golden fixtures under tests/golden/ hold SHA-256 digests produced by the
reference compiled from its sources (tests/golden/make_golden.py):
``zipserv::pack_bf16`` (csrc/HostPacker.h:95-183) and the frozen legacy
encoder (tests/reference_packer.h) for every case of
tests/test_host_packer.cpp:69-111, ``best_exponent_window``
(csrc/CodecUtils.h:40-53) for tests/test_codec_utils.cpp:31-45,
``std::mt19937`` streams, and the CPU bridge ``zipserv_compress``
(integrations/vllm/native/host_bridge.cpp:18-43). No GPU is needed.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def _sha(array) -> str:
    if array is None:
        return hashlib.sha256(b"").hexdigest()
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def packer_golden():
    return json.loads((GOLDEN / "reference_packer.json").read_text())


@pytest.fixture(scope="module")
def codec_golden():
    return json.loads((GOLDEN / "reference_codec.json").read_text())


@pytest.fixture(scope="module")
def bridge_golden():
    return json.loads((GOLDEN / "reference_bridge.json").read_text())


def test_mt19937_streams(oracle_mod, codec_golden):
    for seed, want in codec_golden["mt19937"].items():
        values = oracle_mod.MT19937(int(seed)).take(2000)
        assert values[:16].tolist() == want["first"], seed
        assert oracle_mod.digest(values) == want["sha256_2000"], seed


def test_best_window_trials(oracle_mod, codec_golden):
    """1000 seeded histograms x window widths 1..7 (tests/test_codec_utils.cpp:31-45)."""
    import ctypes

    lib = oracle_mod.lib()
    rng = oracle_mod.MT19937(42).take(1000 * 256)
    for trial, want in enumerate(codec_golden["best_window_trials"]):
        counts = (rng[trial * 256:(trial + 1) * 256] % 10000).astype(np.uint64)
        ptr = counts.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
        got = [lib.oracle_best_window(ptr, width) for width in range(1, 8)]
        assert got == want, trial
    gap = np.zeros(256, dtype=np.uint64)
    gap[50:57] = 2
    gap[120] = gap[126] = 10000
    ptr = gap.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
    assert lib.oracle_best_window(ptr, 7) == codec_golden["best_window_gap_case"]


def test_every_reference_packer_case(oracle_mod, packer_golden):
    """All 296 encoder cases: metadata and the eight buffers byte for byte."""
    seen = 0
    cases = list(oracle_mod.host_packer_cases())
    cases += [(f"decode_mode{i}", w, 256, 256, -1, False)
              for i, w in enumerate(oracle_mod.decode_modes())]
    for name, words, m, k, base, small in cases:
        want = packer_golden[name]
        assert oracle_mod.digest(words) == want["input_sha256"], name
        packed = oracle_mod.pack(words, base, small)
        assert (packed.base, packed.max_common, packed.max_rare) == (
            want["base"], want["max_common"], want["max_rare"]), name
        got = [_sha(b) for b in packed.all_buffers()]
        assert got == want["sha256"], name
        seen += 1
    assert seen == len(packer_golden) == 296


def test_oracle_decode_inverts_every_case(oracle_mod):
    """Independent decode (tests/test_host_packer.cpp:14-44) round-trips every case."""
    for name, words, m, k, base, _small in oracle_mod.host_packer_cases():
        packed = oracle_mod.pack(words, base)
        restored = oracle_mod.decode(packed.abi_buffers(), m, k, packed.start_exp)
        assert np.array_equal(restored, words.reshape(m, k)), name


def test_bridge_cases(oracle_mod, bridge_golden):
    """The C-ABI bridge configuration (base chosen by the encoder, no small
    offsets, start_exp = base - 1) on the seeded Llama-like weights."""
    for label, want in bridge_golden.items():
        w = oracle_mod.llama_weight(want["m"], want["k"], want["seed"], want["outliers"])
        assert oracle_mod.digest(w) == want["input_sha256"], label
        packed = oracle_mod.pack(w)
        bufs = packed.abi_buffers()
        assert [b.size for b in bufs] == want["lengths"], label
        assert [_sha(b) for b in bufs] == want["sha256"], label
        assert (packed.max_common, packed.max_rare, packed.start_exp) == (
            want["max_common"], want["max_rare"], want["start_exp"]), label


def test_exponent_bits_wraps_at_base_zero(oracle_mod):
    """csrc/CodecUtils.h:55-62: uint8(start_exp + code) << 7, wrapping for base 0."""
    lib = oracle_mod.lib()
    assert lib.oracle_exponent_bits(255, 1) == 0
    assert lib.oracle_exponent_bits(255, 7) == 6 << 7
    assert lib.oracle_exponent_bits(115, 1) == 116 << 7
    assert lib.oracle_exponent_bits(248, 7) == 255 << 7


def test_fp32_to_bf16_rounding(oracle_mod):
    """Round-to-nearest-even with quiet NaN, matching __float2bfloat16_rn."""
    lib = oracle_mod.lib()
    vals = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, float("inf"), float("-inf"),
                     1e-40, 0.0, -0.0], dtype=np.float32)
    scalar = np.array([lib.oracle_f32_to_bf16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(scalar, oracle_mod.f32_to_bf16(vals))
    assert scalar[0] == 0x3F80 and scalar[1] == 0x3F80 and scalar[2] == 0x3F81
    nan = oracle_mod.f32_to_bf16(np.array([float("nan")], dtype=np.float32))[0]
    assert (nan & 0x7F80) == 0x7F80 and (nan & 0x7F)
