"""Generate tests/golden/*.json from the reference's own encoder.

Run in a container that has the reference sources (it builds oracle/_ref from
them first):

    python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE_CHECKOUT]

Every digest here comes from the reference compiled from its sources:
``zipserv::pack_bf16`` (csrc/HostPacker.h), the frozen legacy encoder
(tests/reference_packer.h), the CPU C-ABI bridge ``zipserv_compress``
(integrations/vllm/native/host_bridge.cpp), ``best_exponent_window``
(csrc/CodecUtils.h) and ``std::mt19937``. The inputs are the reference tests'
own seeded cases, rebuilt by oracle/oracle.py. The fixtures hold SHA-256
digests and metadata only, so they stay small.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent


class RefPacked(ctypes.Structure):
    _fields_ = [("buffers", ctypes.c_void_p * 8), ("lengths", ctypes.c_uint64 * 8),
                ("tiles", ctypes.c_int32), ("base", ctypes.c_int32),
                ("max_common", ctypes.c_int32), ("max_rare", ctypes.c_int32)]


class NativePacked(ctypes.Structure):  # integrations/vllm/native/host_bridge.h:9-13
    _fields_ = [("buffers", ctypes.c_void_p * 7), ("lengths", ctypes.c_uint64 * 7),
                ("m", ctypes.c_int32), ("k", ctypes.c_int32), ("max_common", ctypes.c_int32),
                ("max_rare", ctypes.c_int32), ("start_exp", ctypes.c_int32)]


def _bytes(ptr, n):
    return ctypes.string_at(ptr, n) if n else b""


def _sha(b: bytes) -> str:
    import hashlib

    return hashlib.sha256(b).hexdigest()


def record(shim, words, m, k, base, small, legacy: bool):
    out = RefPacked()
    words = np.ascontiguousarray(words, dtype=np.uint16)
    assert shim.ref_pack(words.ctypes.data, m, k, base, int(small), 1, ctypes.byref(out)) == 0
    entry = {
        "tiles": out.tiles, "base": out.base, "max_common": out.max_common,
        "max_rare": out.max_rare, "lengths": list(out.lengths),
        "sha256": [_sha(_bytes(out.buffers[i], out.lengths[i])) for i in range(8)],
    }
    shim.ref_free(ctypes.byref(out))
    if legacy:
        leg = RefPacked()
        assert shim.ref_pack_legacy(words.ctypes.data, m, k, entry["base"], ctypes.byref(leg)) == 0
        lsha = [_sha(_bytes(leg.buffers[i], leg.lengths[i])) for i in range(8)]
        shim.ref_free(ctypes.byref(leg))
        # The reference asserts this identity itself (tests/test_host_packer.cpp:61-63).
        for i in range(8):
            if i == 5 and not small:
                continue
            assert lsha[i] == entry["sha256"][i], "legacy and current reference encoders differ"
    return entry


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--ref", default=os.environ.get("ZIPSERV_REFERENCE") or
                        str(ROOT.parent / "reference"),
                        help="reference checkout (default: ZIPSERV_REFERENCE, else a "
                             "`reference` directory beside this repository)")
    args = parser.parse_args()
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all", "ref", f"REF={args.ref}"],
                   check=True)
    shim = ctypes.CDLL(str(ROOT / "oracle/_ref/libref_shim.so"))
    shim.ref_pack.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_uint, ctypes.POINTER(RefPacked)]
    shim.ref_pack_legacy.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(RefPacked)]
    shim.ref_free.argtypes = [ctypes.POINTER(RefPacked)]
    shim.ref_mt_fill.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t]
    shim.ref_best_window.argtypes = [ctypes.c_void_p, ctypes.c_int]

    cases = {}
    for name, words, m, k, base, small in oracle.host_packer_cases():
        cases[name] = {"m": m, "k": k, "base_arg": base, "include_small": small,
                       "input_sha256": oracle.digest(words),
                       **record(shim, words, m, k, base, small, legacy=True)}
    for mode, words in enumerate(oracle.decode_modes()):
        cases[f"decode_mode{mode}"] = {"m": 256, "k": 256, "base_arg": -1, "include_small": False,
                                       "input_sha256": oracle.digest(words),
                                       **record(shim, words, 256, 256, -1, False, legacy=False)}

    mt = {}
    for seed in (42, 12345, 5489):
        buf = np.empty(2000, dtype=np.uint32)
        shim.ref_mt_fill(seed, buf.ctypes.data, buf.size)
        mt[str(seed)] = {"first": buf[:16].tolist(), "sha256_2000": oracle.digest(buf)}

    # tests/test_codec_utils.cpp:31-45: 1000 random histograms x widths 1..7.
    rng_vals = np.empty(1000 * 256, dtype=np.uint32)
    shim.ref_mt_fill(42, rng_vals.ctypes.data, rng_vals.size)
    windows = []
    for trial in range(1000):
        counts = (rng_vals[trial * 256:(trial + 1) * 256] % 10000).astype(np.uint64)
        windows.append([shim.ref_best_window(counts.ctypes.data, w) for w in range(1, 8)])
    gap = np.zeros(256, dtype=np.uint64)
    gap[50:57] = 2
    gap[120] = gap[126] = 10000

    # The C-ABI bridge's own output for the CPU round-trip configuration
    # (the CPU-runnable configuration): 4096x4096 N(0,0.02) seed 0.
    bridge = ctypes.CDLL(str(ROOT / "oracle/_ref/libzipserv_ref_cpu.so"))
    bridge.zipserv_compress.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(NativePacked)]
    bridge.zipserv_free.argtypes = [ctypes.POINTER(NativePacked)]
    abi = {}
    for label, (m, k, seed, outl) in {"c1_4096x4096": (4096, 4096, 0, 0.0),
                                      "o_proj_small_256x512": (256, 512, 3, 0.0),
                                      "stress_1024x2048": (1024, 2048, 7, 0.05)}.items():
        w = oracle.llama_weight(m, k, seed, outl)
        nat = NativePacked()
        assert bridge.zipserv_compress(w.ctypes.data, m, k, ctypes.byref(nat)) == 0
        abi[label] = {"m": m, "k": k, "seed": seed, "outliers": outl,
                      "input_sha256": oracle.digest(w),
                      "lengths": list(nat.lengths), "max_common": nat.max_common,
                      "max_rare": nat.max_rare, "start_exp": nat.start_exp,
                      "storage_bytes": int(sum(nat.lengths)),
                      "sha256": [_sha(_bytes(nat.buffers[i], nat.lengths[i])) for i in range(7)]}
        bridge.zipserv_free(ctypes.byref(nat))

    (OUT / "reference_packer.json").write_text(json.dumps(cases, indent=0, sort_keys=True) + "\n")
    (OUT / "reference_codec.json").write_text(json.dumps(
        {"mt19937": mt, "best_window_trials": windows,
         "best_window_gap_case": shim.ref_best_window(gap.ctypes.data, 7)},
        separators=(",", ":")) + "\n")
    (OUT / "reference_bridge.json").write_text(json.dumps(abi, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(cases)} packer cases, {len(abi)} bridge cases")


if __name__ == "__main__":
    main()
