"""Host-side planning for the BF16 ZipGEMM path (CPU only).

Mirrors ``zipserv_vllm.bf16_policy`` (integrations/vllm/zipserv_vllm/
bf16_policy.py:14-134): the same names, dataclasses, argument meaning and
rejection messages' purpose, so the linear method can call either. What is
specific to this B200 library:

* The fused kernel schedules K itself (a persistent grid whose CTAs take
  equal ranges of K slices; split row blocks are summed in FP32 inside the
  kernel, in a fixed order), so ``split_k`` never needs a caller workspace:
  candidates carry ``workspace_bytes = 0``. The split the planner returns
  satisfies the native contract and is passed through; the kernel's own
  schedule does not depend on it.
* Scores model the reference's split choice on this kernel's cost shape: one
  CTA per SM, a 128-row block per CTA, N tiles of up to 128 tokens, and a
  fixed start-up cost of about three K slices per CTA (measured on B200: ~3 us
  set-up against ~0.85 us per K slice per SM).

Limits (``gemm_rejection``) follow csrc/CodecUtils.h:11-36 exactly: they are
the contract the native entry points validate.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

INT32_MAX = 2**31 - 1
GRID_Y_MAX = 65535
MAX_CLUSTER = 16          # largest explicit K partition the native API accepts
STARTUP_SLICES = 3.0      # per-CTA fixed cost, in K-slice units (B200 measurement)


# Token count above which decode + stock GEMM beats the fused kernel on a
# B200, measured for the Llama-3-8B linears (per-call device time summed over
# qkv, o, gate_up and down, cold L2): the fused kernel wins at 128 tokens,
# decode + GEMM at 192 and above; small-M layers (qkv, o) cross near 128,
# gate_up near 320. Use it as large_batch_tokens when running eagerly or with
# CUDA-graph capture sizes within it.
B200_LARGE_BATCH_TOKENS = 176

# Per-weight crossover on a B200: the first token count at which
# decompression + cuBLAS BF16 beats the fused kernel, per weight size (M*K
# elements), measured with per-call device time after an L2 flush
# (bench.py --threshold-sweep; token counts 16 .. 768): Llama-3-8B o (16.8M)
# crosses at 32, qkv (25.2M) at 128, down (58.7M) at 256, gate_up (117M) at
# 384; Llama-3-70B TP-1 o (67.1M) at 256, qkv (83.9M), down and gate_up at
# 384. A weight above the last bound uses its value.
B200_CROSSOVER = (
    (20_000_000, 32),
    (40_000_000, 128),
    (70_000_000, 256),
    (float("inf"), 384),
)


def b200_token_limit(m: int, k: int) -> int:
    """Largest token count the fused kernel should serve for an m x k weight
    on a B200 (one below the measured crossover)."""
    elements = m * k
    for bound, crossover in B200_CROSSOVER:
        if elements <= bound:
            return crossover - 1
    return B200_CROSSOVER[-1][1] - 1


@dataclass(frozen=True)
class DispatchSettings:
    """Dispatch knobs (reference ``DispatchSettings``): ``fixed`` uses the
    configured split, ``tokens`` / ``shape`` plan per call and send batches
    above ``large_batch_tokens`` to decode + stock GEMM."""

    mode: str = "fixed"
    # The reference's default. On a B200, B200_LARGE_BATCH_TOKENS is faster
    # (see there); it is not the default because planned dispatch with
    # full-decode CUDA graphs needs every capture size within this threshold.
    large_batch_tokens: int = 768
    workspace_bytes: int = 64 * 2**20
    partial_dtype: str = "bf16"
    decode_workspace_bytes: int = 256 * 2**20
    # Also cap each layer at its measured B200 crossover (b200_token_limit),
    # so small layers switch to decompression + stock GEMM sooner than large
    # ones.
    per_shape_threshold: bool = False

    def __post_init__(self):
        if self.mode not in ("fixed", "tokens", "shape"):
            raise ValueError("dispatch must be fixed, tokens or shape")
        if self.partial_dtype not in ("bf16", "fp32"):
            raise ValueError("partial_dtype must be bf16 or fp32")
        for name in ("large_batch_tokens",):
            value = getattr(self, name)
            if type(value) is not int or value < 1:
                raise ValueError(f"{name} must be a positive integer")
        if type(self.per_shape_threshold) is not bool:
            raise ValueError("per_shape_threshold must be true or false")
        for name in ("workspace_bytes", "decode_workspace_bytes"):
            value = getattr(self, name)
            if type(value) is not int or value < 0:
                raise ValueError(f"{name} must be a nonnegative integer")


def gemm_rejection(m: int, tokens: int, k: int, split_k: int) -> str | None:
    """The native GEMM contract evaluated with exact host integers, before
    any allocation (csrc/CodecUtils.h:19-36)."""
    if any(type(v) is not int for v in (m, tokens, k, split_k)):
        return "GEMM dimensions and Split-K must be integers"
    if m <= 0 or k <= 0 or m % 64 or k % 64 or tokens < 0:
        return "Require positive 64-aligned weight dimensions and nonnegative tokens"
    if split_k < 1 or (k // 64) % split_k:
        return "Split-K must divide the number of 64-column weight tiles"
    if max(m * tokens * split_k, k * tokens, m * k) > INT32_MAX:
        return "Output, activations or Split-K workspace exceed native int32 indexing"
    if (m // 64) * split_k > GRID_Y_MAX:
        return "Split-K exceeds CUDA grid.y"
    return None


def startup_rejection(m: int, k: int, split_k: int, max_tokens: int | None) -> str | None:
    """Reason to keep a layer dense for its planned maximum batch, or None."""
    if type(max_tokens) is not int or max_tokens <= 0:
        return "A positive scheduler max_num_batched_tokens is required for compression planning"
    reason = gemm_rejection(m, max_tokens, k, split_k)
    if reason:
        return reason
    if m * k > INT32_MAX - 4096:
        return "Weight packing exceeds the native int32 offset bound"
    return None


def decode_budget_rejection(m: int, k: int, settings: DispatchSettings) -> str | None:
    """Dynamic dispatch decodes whole weights for large batches: reject
    weights whose BF16 copy exceeds the decode budget."""
    if settings.mode != "fixed" and m * k * 2 > settings.decode_workspace_bytes:
        return (f"Decoded BF16 weight requires {m * k * 2} bytes, exceeding the "
                f"decode_workspace_bytes budget of {settings.decode_workspace_bytes}")
    return None


@dataclass(frozen=True)
class SplitCandidate:
    split_k: int
    blocks: int
    workspace_bytes: int
    score: float


def token_tile(tokens: int) -> int:
    """N tile of the fused kernel: a multiple of 16 up to 128 tokens."""
    return max(16, min(128, (tokens + 15) // 16 * 16))


@lru_cache(maxsize=4096)
def split_candidates(m: int, tokens: int, k: int, sms: int, workspace_bytes: int,
                     partial_bytes: int = 2) -> tuple[SplitCandidate, ...]:
    """Every admissible split (a divisor of K/64 up to 16, so the native
    Split-K contract holds) with its wave-model score (lower is better):
    waves x (K slices per CTA + start-up). The kernel reduces K ranges
    internally, so no caller workspace is used."""
    if type(sms) is not int or sms < 1 or partial_bytes not in (2, 4):
        raise ValueError("Require positive SM count and 2- or 4-byte partials")
    if type(workspace_bytes) is not int or workspace_bytes < 0:
        raise ValueError("workspace_bytes must be a nonnegative integer")
    if gemm_rejection(m, tokens, k, 1):
        return ()
    slices = k // 64
    row_blocks = (m // 64 + 1) // 2
    n_tiles = max(1, -(-max(tokens, 1) // token_tile(tokens)))
    out = []
    for split in range(1, min(MAX_CLUSTER, slices) + 1):
        if slices % split or gemm_rejection(m, tokens, k, split):
            continue
        ctas = row_blocks * n_tiles * split
        slots = (sms // split) * split  # whole split groups per wave
        if slots == 0:
            continue
        waves = -(-ctas // slots)
        per_cta = -(-slices // split) + STARTUP_SLICES + (1.0 if split > 1 else 0.0)
        out.append(SplitCandidate(split, ctas, 0, waves * per_cta))
    return tuple(out)


def fused_token_limit(m: int, k: int, settings: DispatchSettings) -> int:
    """Largest batch the planner sends to the fused kernel for an m x k weight."""
    if settings.per_shape_threshold:
        return min(settings.large_batch_tokens, b200_token_limit(m, k))
    return settings.large_batch_tokens


@lru_cache(maxsize=4096)
def select_split(m: int, tokens: int, k: int, sms: int, settings: DispatchSettings,
                 fixed_split: int = 1) -> int | None:
    """The split to request, or None for decode + stock GEMM (large batches)."""
    if settings.mode == "fixed":
        return fixed_split
    if tokens > fused_token_limit(m, k, settings):
        return None
    candidates = split_candidates(m, tokens, k, sms, settings.workspace_bytes,
                                  4 if settings.partial_dtype == "fp32" else 2)
    if not candidates:
        return None
    if settings.mode == "tokens":
        desired = 8 if tokens <= 32 else 4 if tokens <= 128 else 1
        return max(c.split_k for c in candidates if c.split_k <= desired)
    return min(candidates, key=lambda c: (c.score, c.split_k)).split_k
