"""Test helpers: move oracle/ABI packed data to torch, compare GEMM outputs."""
from __future__ import annotations

import numpy as np
import torch

from zipserv_asplos26_b200 import runtime


def make_packed(oracle_packed, m: int, k: int) -> runtime.PackedWeight:
    """Wrap an oracle.OraclePacked (CPU, any window) as a PackedWeight."""
    bufs = tuple(torch.from_numpy(np.ascontiguousarray(b).view(np.uint8).copy())
                 for b in oracle_packed.abi_buffers())
    return runtime.PackedWeight(bufs, m, k, oracle_packed.max_common, oracle_packed.max_rare,
                                oracle_packed.start_exp)


def bf16_tensor(words: np.ndarray) -> torch.Tensor:
    """uint16 BF16 bit patterns -> torch.bfloat16 (CPU)."""
    return torch.from_numpy(np.ascontiguousarray(words, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def words_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def rel_errors(actual_bits: np.ndarray, expected_bits: np.ndarray) -> tuple[float, float]:
    """(max |a-e| / max |e|, mean |a-e| / mean |e|) over BF16 outputs as floats.

    Tolerance used by the parity tests (from the hot path's specification):
    max <= 1e-2 and mean <= 1e-3 against the FP32-accumulated oracle on the
    identical decoded weights."""
    a = (actual_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    e = (expected_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    d = np.abs(a - e)
    scale_max = max(np.abs(e).max(), 1e-30)
    scale_mean = max(np.abs(e).mean(), 1e-30)
    return float(d.max() / scale_max), float(d.mean() / scale_mean)


MAX_REL_TOL = 1e-2
MEAN_REL_TOL = 1e-3
