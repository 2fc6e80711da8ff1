"""Tensor-parallel host logic on two and four CPU ranks (gloo): shard boundaries,
per-rank packing of its own shard, column outputs concatenating to the full
product and row partials all-reduced to it. The per-rank multiply is the
CPU oracle (decode + FP32 GEMM) standing in for the CUDA kernel, so the test
checks the decomposition and the collective, not the kernel.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zipserv_asplos26_b200 import runtime, tp

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_linear(x: torch.Tensor, packed) -> torch.Tensor:
    """x [N, K] BF16 -> FP32 [N, M] from the packed shard (CPU oracle)."""
    from oracle import oracle

    bufs = [b.numpy() for b in packed.buffers]
    w = oracle.decode(bufs, packed.m, packed.k, packed.start_exp)
    xw = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    _, yf = oracle.gemm(w, xw)
    return torch.from_numpy(yf.copy())


def _weights(m, k, n):
    g = torch.Generator().manual_seed(m + k)
    w = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16)
    return w, x


def _rank_main(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle

        oracle.ensure_built()
        out = {}
        for kind, (m, k) in (("column", (256, 384)), ("row", (192, 512))):
            w, x = _weights(m, k, 5)
            layer = tp.ParallelLinear.from_weight(w, kind, world, rank, "cpu")
            y = layer.forward(x, linear=_oracle_linear)
            if kind == "column":
                parts = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(parts, y)
                y = torch.cat(parts, dim=-1)
            full = _oracle_linear(x, runtime.compress(w))
            out[kind] = float((y - full).abs().max() / full.abs().max())
            out[kind + "_local_k"] = layer.packed.k
            out[kind + "_local_m"] = layer.packed.m
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_column_and_row_parallel(native_lib, oracle_mod, world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        res = results[r]
        # Column: every rank's M/world rows concatenate to the full product exactly.
        assert res["column"] == 0.0 and res["column_local_m"] == 256 // world
        # Row: FP32 partial sums reordered by the K split only.
        assert res["row"] < 1e-5 and res["row_local_k"] == 512 // world
        assert res["row_local_m"] == 192


def test_shard_bounds_reject_unaligned_splits():
    assert tp.shard_bounds(4096, 8, 3) == (1536, 2048)
    with pytest.raises(ValueError):
        tp.shard_bounds(4096, 3, 0)
    with pytest.raises(ValueError):
        tp.shard_bounds(192, 2, 0)   # 96 per shard is not 64-aligned
    with pytest.raises(ValueError):
        tp.shard_bounds(128, 2, 2)
    w = torch.zeros(256, 512, dtype=torch.bfloat16)
    assert tuple(tp.shard_weight(w, "column", 2, 1).shape) == (128, 512)
    assert tuple(tp.shard_weight(w, "row", 4, 0).shape) == (256, 128)
    with pytest.raises(ValueError):
        tp.shard_weight(w, "diagonal", 2, 0)
