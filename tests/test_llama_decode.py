"""The Llama-3 decode-step workload (zipserv_asplos26_b200.llama_decode, the
benchmarked decode-step model) at a reduced shape.

CPU (gloo, two and four ranks): the Megatron split of the step — qkv by heads,
gate_up by intermediate rows, o and down on K with an all-reduce, the
lm_head by vocabulary rows with a padded last shard — reproduces the
single-rank logits and greedy tokens of the same seeded model (dense
weights, so the test checks the decomposition and collectives).
GPU: the same model with every linear packed on the GPU and run by the
fused kernel gives the dense model's logits within the hot path's GEMM
tolerance, and a CUDA-graph replay of the step equals the eager step.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zipserv_asplos26_b200.llama_decode import DecodeStep, LlamaShape

SMALL = LlamaShape(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=32, ffn=512,
                   vocab=1000, context=64)
# Four KV heads so the heads split four ways (the benchmarked model has 8 KV
# heads, which split up to TP 8).
SMALL4 = LlamaShape(layers=2, hidden=256, heads=8, kv_heads=4, head_dim=32, ffn=512,
                    vocab=1000, context=64)
TOKENS = [3, 141, 592, 653, 589, 793]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results, shape=SMALL):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        model = DecodeStep(shape, len(TOKENS), "cpu", mode="dense", world=world, rank=rank)
        tokens = torch.tensor(TOKENS)
        logits = model.logits(tokens)
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits)
        # the step issues its own collectives; every rank takes part
        nxt = model.step(tokens)
        if rank == 0:
            results[world] = (torch.cat(parts, dim=1)[:, :shape.vocab], nxt)
    finally:
        dist.destroy_process_group()


def _run(world, shape=SMALL):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), results, shape), nprocs=world,
                       start_method="spawn", join=True)
    return results[world]


@pytest.mark.parametrize("world,shape", [(2, SMALL), (4, SMALL4)])
def test_tensor_parallel_step_matches_one_rank(world, shape):
    one_logits, one_next = _run(1, shape)
    tp_logits, tp_next = _run(world, shape)
    scale = one_logits.abs().max()
    assert (tp_logits - one_logits).abs().max() / scale < 2e-2
    # Greedy tokens agree wherever the top-2 margin exceeds the rounding noise.
    top2 = one_logits.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 5e-2 * scale
    assert clear.any()
    assert torch.equal(one_next[clear], tp_next[clear])


@pytest.mark.gpu
def test_zipgemm_step_matches_dense_and_replays_in_a_graph(native_lib):
    from helpers import MAX_REL_TOL

    from zipserv_asplos26_b200 import runtime

    zip_model = DecodeStep(SMALL, len(TOKENS), "cuda", mode="zipgemm")
    dense = DecodeStep(SMALL, len(TOKENS), "cuda", mode="dense")
    assert zip_model.weight_bytes() < dense.weight_bytes()
    tokens = torch.tensor(TOKENS, device="cuda")
    a, b = zip_model.logits(tokens), dense.logits(tokens)
    real = torch.isfinite(b)
    assert (a[real] - b[real]).abs().max() / b[real].abs().max() <= 4 * MAX_REL_TOL
    eager = zip_model.step(tokens)
    graph, out = zip_model.capture(tokens)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert runtime.device_flags() == 0
