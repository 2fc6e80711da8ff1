"""The GPU encoder (runtime.compress_device, C ABI zipserv_pack_device_*):
byte-identical to the reference encoder on every golden case the
reference's own packer tests hold (tests/test_host_packer.cpp:69-111 and the
bridge cases, digests recorded from the reference built here), and equal to
the host encoder on full-size weights, which then decode bit-exactly.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import bf16_tensor
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()


def test_every_reference_packer_case(native_lib, oracle_mod):
    golden = json.loads((GOLDEN / "reference_packer.json").read_text())
    seen = 0
    cases = [(name, words, base) for name, words, _m, _k, base, _s in oracle_mod.host_packer_cases()]
    cases += [(f"decode_mode{i}", w, -1) for i, w in enumerate(oracle_mod.decode_modes())]
    for name, words, base_arg in cases:
        want = golden[name]
        # base_arg -1 lets the encoder choose the window (the reference's
        # choice is recorded as want["base"]); otherwise the window is fixed.
        packed = runtime.compress_device(bf16_tensor(words).cuda(),
                                         base=want["base"] if base_arg >= 0 else -1)
        assert packed.start_exp == (want["base"] - 1) % 256, name
        assert (packed.max_common, packed.max_rare) == (want["max_common"], want["max_rare"]), name
        # Reference digests: sm, rare, b1, b2, b3, small offsets, medium, global.
        for got, idx in zip(packed.buffers, (0, 1, 2, 3, 4, 6, 7)):
            assert _sha(got) == want["sha256"][idx], (name, idx)
        seen += 1
    assert seen == len(golden)


def test_reference_bridge_cases(native_lib, oracle_mod):
    golden = json.loads((GOLDEN / "reference_bridge.json").read_text())
    for label, want in golden.items():
        w = oracle_mod.llama_weight(want["m"], want["k"], want["seed"], want["outliers"])
        packed = runtime.compress_device(bf16_tensor(w).cuda())
        assert list(packed.lengths) == want["lengths"], label
        assert [_sha(b) for b in packed.buffers] == want["sha256"], label
        assert (packed.m, packed.k, packed.max_common, packed.max_rare, packed.start_exp) == (
            want["m"], want["k"], want["max_common"], want["max_rare"], want["start_exp"])


@pytest.mark.parametrize("m,k,outliers", [(28672, 4096, 0.0), (4096, 14336, 0.0),
                                          (28672, 8192, 0.05), (64, 4096, 0.0),
                                          (4096, 64, 0.3)])
def test_full_size_equals_host_encoder_and_decodes(native_lib, oracle_mod, m, k, outliers):
    w = oracle_mod.llama_weight(m, k, seed=m + k, outliers=outliers)
    dev = bf16_tensor(w).cuda()
    on_gpu = runtime.compress_device(dev)
    on_host = runtime.compress(bf16_tensor(w))
    assert (on_gpu.max_common, on_gpu.max_rare, on_gpu.start_exp) == (
        on_host.max_common, on_host.max_rare, on_host.start_exp)
    for a, b in zip(on_gpu.buffers, on_host.buffers):
        assert torch.equal(a.cpu(), b)
    assert torch.equal(runtime.decompress(on_gpu).view(torch.int16), dev.view(torch.int16))
    assert runtime.device_flags() == 0


def test_special_values_and_argument_checks(native_lib):
    words = np.array([0, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x0001, 0x3F80, 0xBF80], np.uint16)
    mat = np.tile(words, 64 * 64 // 8).reshape(64, 64)
    got = runtime.compress_device(bf16_tensor(mat).cuda())
    want = runtime.compress(bf16_tensor(mat))
    assert all(torch.equal(a.cpu(), b) for a, b in zip(got.buffers, want.buffers))
    with pytest.raises(ValueError):
        runtime.compress_device(torch.zeros(64, 64, dtype=torch.bfloat16))  # host tensor
    with pytest.raises(ValueError):
        runtime.compress_device(torch.zeros(96, 64, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        runtime.compress_device(torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda"), base=250)
