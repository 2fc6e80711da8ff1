"""The fused row-parallel all-reduce (zipserv_mm_allreduce through
tp.PeerExchange) on two or more GPUs of one node: each rank multiplies its K
shard of the o-projection and down-projection weights and receives the full
sum over ranks from the same kernel.

Checked per token count (including split row blocks of the default
schedule): every rank stores bit-identical outputs, the sum matches an FP32
product of the full, bit-exactly decoded weight within the hot path's
tolerance, repeated calls are deterministic, a CUDA-graph replay (the
launch counter lives on the device) equals the eager call, and no wait gives
up. Runs as child processes, one per GPU (NCCL only for setup and checks);
skipped with fewer than two GPUs.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = (("o", 4096, 4096), ("down", 4096, 14336))
TOKENS = (1, 16, 64, 128)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from helpers import rel_errors, words_of
    from zipserv_asplos26_b200 import runtime, tp

    out = {"errors": [], "identical": True, "deterministic": True, "graph": True}
    exchange = tp.PeerExchange(4096, 128)
    exchange.fused_max_tokens = 128  # the fused kernel at every tested token count
    try:
        for li, (name, m, k) in enumerate(SHAPES):
            g = torch.Generator().manual_seed(50 + li)
            w = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
            layer = tp.ParallelLinear.from_weight(w, tp.ROW, world, rank, "cuda")
            w_dev = w.cuda()
            for n in TOKENS:
                x = torch.randn(n, k, generator=torch.Generator().manual_seed(n)).to(
                    torch.bfloat16).cuda()
                y = layer.forward(x, exchange=exchange)
                again = layer.forward(x, exchange=exchange)
                torch.cuda.synchronize()
                out["deterministic"] &= torch.equal(y.view(torch.int16), again.view(torch.int16))
                gathered = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(gathered, y)
                out["identical"] &= all(torch.equal(t.view(torch.int16), y.view(torch.int16))
                                        for t in gathered)
                prev = torch.backends.cuda.matmul.allow_tf32
                torch.backends.cuda.matmul.allow_tf32 = False
                ref = (x.float() @ w_dev.float().t()).to(torch.bfloat16)
                torch.backends.cuda.matmul.allow_tf32 = prev
                mx, mean = rel_errors(words_of(y), words_of(ref))
                out["errors"].append((name, n, mx, mean))
                # The other route (GEMM + NCCL all-reduce), as chosen above
                # the default token limit.
                c0, c1 = tp.shard_bounds(k, world, rank)
                y2 = exchange.linear(x[..., c0:c1].contiguous(), layer.packed, fused=False)
                mx, mean = rel_errors(words_of(y2), words_of(ref))
                out["errors"].append((name + "+nccl", n, mx, mean))
            # CUDA graph of the fused call (shape never captured before).
            x = torch.randn(16, k, generator=torch.Generator().manual_seed(99)).to(
                torch.bfloat16).cuda()
            eager = layer.forward(x, exchange=exchange)
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    captured = layer.forward(x, exchange=exchange)
            torch.cuda.current_stream().wait_stream(stream)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            out["graph"] &= torch.equal(captured.view(torch.int16), eager.view(torch.int16))
            del graph
        out["flags"] = runtime.device_flags()
    finally:
        exchange.close()
        dist.destroy_process_group()
    results[rank] = out


def test_fused_row_parallel_allreduce():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn", join=True)
    from helpers import MAX_REL_TOL, MEAN_REL_TOL

    assert sorted(results.keys()) == list(range(world))
    for rank, out in results.items():
        assert out["flags"] == 0, rank
        assert out["identical"] and out["deterministic"] and out["graph"], (rank, out)
        for name, n, mx, mean in out["errors"]:
            # The NCCL route sums BF16 partial outputs (each rank's GEMM rounds
            # to BF16, then the all-reduce adds in BF16): three roundings where
            # the fused kernel has one, so it gets three times the tolerance.
            scale = 3.0 if name.endswith("+nccl") else 1.0
            assert mx <= scale * MAX_REL_TOL and mean <= scale * MEAN_REL_TOL, (
                rank, name, n, mx, mean)
