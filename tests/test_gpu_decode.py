"""Bit-exact GPU decompression (zipserv_decode through the C ABI) against the
original words and the CPU oracle. Cases follow the reference's own tests:
tests/test_cuda.cu:96-107 (all words and edge modes) and the encoder cases of
tests/test_host_packer.cpp:69-111, plus benchmark-sized weights."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import bf16_tensor, make_packed, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu


def decode_gpu(packed: runtime.PackedWeight) -> np.ndarray:
    out = runtime.decompress(packed.to("cuda"))
    torch.cuda.synchronize()
    assert runtime.device_flags() == 0
    return words_of(out)


@pytest.mark.parametrize("mode", range(4))
def test_all_words_and_edge_modes(native_lib, oracle_mod, mode):
    words = oracle_mod.decode_modes()[mode]
    packed = runtime.compress(bf16_tensor(words))
    assert np.array_equal(decode_gpu(packed), words)


def test_reference_encoder_cases(native_lib, oracle_mod):
    """Every window base 0..249, constants, padding boundaries, odd shapes,
    mixed empty/full tiles: GPU decode of the oracle's (== reference's) packing."""
    checked = 0
    for name, words, m, k, base, _small in oracle_mod.host_packer_cases():
        p = oracle_mod.pack(words, base)
        got = decode_gpu(make_packed(p, m, k))
        assert np.array_equal(got, words), name
        checked += 1
    assert checked == 292


@pytest.mark.parametrize("shape,outliers", [((4096, 4096), 0.0), ((1024, 2048), 0.05),
                                            ((64, 192), 0.0), ((192, 64), 0.3)])
def test_weight_matrices(native_lib, oracle_mod, shape, outliers):
    m, k = shape
    words = oracle_mod.llama_weight(m, k, seed=11, outliers=outliers)
    packed = runtime.compress(bf16_tensor(words))
    assert np.array_equal(decode_gpu(packed), words)


def test_decode_into_strided_destination_rejected_and_aligned_ok(native_lib, oracle_mod):
    words = oracle_mod.llama_weight(128, 128, seed=3)
    packed = runtime.compress(bf16_tensor(words)).to("cuda")
    base = torch.empty(128 * 128 + 8, dtype=torch.bfloat16, device="cuda")
    lib = runtime._cuda_library()
    stream = torch.cuda.current_stream().cuda_stream
    args = [b.data_ptr() for b in packed.buffers]
    misaligned = base.data_ptr() + 2
    assert lib.zipserv_decode(stream, *args, packed.max_common, packed.max_rare,
                              packed.start_exp, misaligned, 128, 128) == 1
    assert lib.zipserv_decode(stream, *args, packed.max_common, packed.max_rare,
                              packed.start_exp, base.data_ptr() + 16, 128, 128) == 0
    torch.cuda.synchronize()
    assert np.array_equal(words_of(base[8:]).reshape(128, 128), words)


@pytest.mark.parametrize("m,k,outliers", [(64, 64, 0.0), (128, 6400, 0.0), (2368, 1024, 0.0),
                                          (9472, 384, 0.02), (4160, 2112, 0.1)])
def test_chunk_schedules(native_lib, oracle_mod, m, k, outliers):
    """Chunk counts below, at and a few times the persistent grid (one chunk,
    fewer chunks than CTAs, 2-3 chunks per CTA, uneven tails), with payload
    capacities that change the slot ring: every producer drains its last
    copies and no bounded wait gives up."""
    words = oracle_mod.llama_weight(m, k, seed=5, outliers=outliers)
    packed = runtime.compress(bf16_tensor(words))
    assert np.array_equal(decode_gpu(packed), words)
