"""Megatron-style tensor parallelism for compressed linears (one process per
GPU, ``torch.distributed`` over NCCL for the plumbing).

Column-parallel layers (qkv, gate_up) split W by output rows: every rank
packs and multiplies its own [M/tp, K] shard and produces [N, M/tp] with no
collective. Row-parallel layers (o, down) split W by K: every rank packs its
[M, K/tp] shard, multiplies the matching K/tp slice of the activations and the
[N, M] partial outputs are summed across ranks: either with an NCCL
all-reduce after the GEMM, or inside the GEMM kernel itself (``PeerExchange``:
each CTA stores its finished FP32 output pieces into every rank's receive
buffer over NVLink and sums the ranks' pieces, see zipserv_mm_allreduce).
Every rank packs its own shard, so each has its own exponent window and
packed maxima. Shards must stay 64-aligned (M/tp and K/tp multiples of 64).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from . import runtime

COLUMN, ROW = "column", "row"


def shard_bounds(size: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's equal share of `size`; shares must be 64-aligned."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if size % world or (size // world) % 64:
        raise ValueError(f"{size} does not split into {world} shards that are multiples of 64")
    share = size // world
    return rank * share, (rank + 1) * share


def shard_weight(weight: Tensor, kind: str, world: int, rank: int) -> Tensor:
    """This rank's contiguous shard of an [M, K] weight."""
    m, k = weight.shape
    if kind == COLUMN:
        r0, r1 = shard_bounds(m, world, rank)
        return weight[r0:r1].contiguous()
    if kind == ROW:
        c0, c1 = shard_bounds(k, world, rank)
        return weight[:, c0:c1].contiguous()
    raise ValueError("kind must be 'column' or 'row'")


class PeerExchange:
    """Receive buffers, flags and launch counter for the fused row-parallel
    all-reduce, shared by the ranks of a process group through CUDA IPC and
    sized for outputs up to [max_tokens, max_m]. Create it on every rank (it
    exchanges handles with a collective) and close it on every rank."""

    def __init__(self, max_m: int, max_tokens: int, group=None,
                 device: torch.device | None = None) -> None:
        lib = runtime._cuda_library()
        if not hasattr(lib, "zipserv_mm_allreduce"):
            raise RuntimeError("This ZipServ library has no fused all-reduce")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.max_m, self.max_tokens = max_m, max_tokens
        rb, fb = ctypes.c_uint64(0), ctypes.c_uint64(0)
        runtime._check(lib.zipserv_mm_allreduce_sizes(max_m, max_tokens, self.world,
                                                      ctypes.byref(rb), ctypes.byref(fb)))
        self.recv_bytes, self.flag_bytes = int(rb.value), int(fb.value)
        self._owned: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            recv, flags, state = (self._alloc(n) for n in (self.recv_bytes, self.flag_bytes, 16))
            mine = []
            for ptr in (recv, flags):
                h = (ctypes.c_char * 64)()
                runtime._check(lib.zipserv_ipc_handle(ctypes.c_void_p(ptr), h))
                mine.append(bytes(h))
            handles: list = [None] * self.world
            dist.all_gather_object(handles, mine, group=group)
            self.recv = (ctypes.c_void_p * self.world)()
            self.flags = (ctypes.c_void_p * self.world)()
            for r, (hr, hf) in enumerate(handles):
                if r == self.rank:
                    self.recv[r], self.flags[r] = recv, flags
                    continue
                self.recv[r], self.flags[r] = self._open(hr), self._open(hf)
            self.state = state
        dist.barrier(group=group)

    def _alloc(self, nbytes: int) -> int:
        ptr = ctypes.c_void_p()
        runtime._check(runtime._cuda_library().zipserv_ipc_alloc(nbytes, ctypes.byref(ptr)))
        self._owned.append(ptr.value)
        return ptr.value

    def _open(self, handle: bytes) -> int:
        ptr = ctypes.c_void_p()
        runtime._check(runtime._cuda_library().zipserv_ipc_open(handle, ctypes.byref(ptr)))
        self._opened.append(ptr.value)
        return ptr.value

    # Largest token count for which `linear` uses the fused kernel by default.
    # Measured on B200 (TP 2, Llama-3-8B o and down shards, per-call device
    # time): fused 29 vs 34 us (o) and 38 vs 41 us (down) at 1 token, still
    # ahead at 32, behind at 64 and 128, where the kernel's collect (one
    # polling round per rank and 16-column chunk, on the four epilogue warps)
    # costs more than NCCL's all-reduce.
    fused_max_tokens = 32

    def linear(self, x: Tensor, packed: runtime.PackedWeight, out: Tensor | None = None,
               fused: bool | None = None) -> Tensor:
        """sum over ranks of x_r @ W_r^T for this rank's K shard: [.., K/tp] -> [.., M].

        `fused` None: the fused kernel up to `fused_max_tokens` tokens, above
        it the GEMM followed by an all-reduce over the group (every rank makes
        the same choice, as it passes the same token count); True / False
        force one route."""
        m, k = packed.m, packed.k
        if x.dtype != torch.bfloat16 or x.shape[-1] != k or x.device != self.device:
            raise ValueError("ZipServ linear requires BF16 activations with the matching input width")
        n = x.numel() // k
        if m > self.max_m or n > self.max_tokens:
            raise ValueError("output exceeds the exchange buffers' size")
        flat = x.reshape(n, k).contiguous()
        if out is None:
            out = x.new_empty((n, m))
        if n and not (n <= self.fused_max_tokens if fused is None else fused):
            runtime.linear_kparts(flat, packed, 0, out=out.view(n, m))
            dist.all_reduce(out, group=self.group)
        elif n:
            lib = runtime._cuda_library()
            runtime._check(lib.zipserv_mm_allreduce(
                torch.cuda.current_stream(self.device).cuda_stream,
                *(b.data_ptr() for b in packed.buffers), packed.max_common, packed.max_rare,
                packed.start_exp, flat.data_ptr(), out.data_ptr(), m, n, k, self.world, self.rank,
                self.recv, self.flags, ctypes.c_void_p(self.state), self.recv_bytes,
                self.flag_bytes))
        return out.reshape(*x.shape[:-1], m)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier, so
        no rank still writes into them)."""
        if not self._owned and not self._opened:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = runtime._cuda_library()
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                lib.zipserv_ipc_close(ctypes.c_void_p(ptr))
            for ptr in self._owned:
                lib.zipserv_ipc_free(ctypes.c_void_p(ptr))
        self._owned, self._opened = [], []


@dataclass
class ParallelLinear:
    """One rank's part of a tensor-parallel compressed linear."""

    packed: runtime.PackedWeight
    kind: str
    world: int
    rank: int
    group: object = None

    @classmethod
    def from_weight(cls, weight: Tensor, kind: str, world: int, rank: int,
                    device: torch.device | str, group=None) -> "ParallelLinear":
        shard = shard_weight(weight, kind, world, rank)
        return cls(runtime.compress(shard).to(device), kind, world, rank, group)

    def forward(self, x: Tensor, linear=None, exchange: PeerExchange | None = None) -> Tensor:
        """Column: x [.., K] -> [.., M/tp]. Row: x [.., K] (full width; the
        rank takes its K slice) -> [.., M], summed over the group: inside the
        kernel when an `exchange` is given, else with an all-reduce.
        `linear` defaults to runtime.linear."""
        linear = runtime.linear if linear is None else linear
        if self.kind == COLUMN:
            return linear(x, self.packed)
        c0, c1 = shard_bounds(x.shape[-1], self.world, self.rank)
        shard = x[..., c0:c1].contiguous()
        if exchange is not None and self.world > 1:
            return exchange.linear(shard, self.packed)
        y = linear(shard, self.packed)
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y
