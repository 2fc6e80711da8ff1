"""The fused kernel's in-kernel K reduction under the conditions that decide
its route, and its scratch under stream capture.

* Forcing the last-arrival route (reducer wait 0) gives outputs identical
  bit for bit to the waiting reducer: both sum the K parts in the same order
  (replaces csrc/Reduction_Kernel.cuh:16-41 of the reference, whose separate
  kernel sums [split_k, n, m] partials).
* A fused GEMM launched while a long decompression on another stream holds
  every SM (its CTAs start late and at different times) still gives the
  exact result of a solo run, and no wait gives up.
* A shape that needs K-range scratch is captured in a CUDA graph on a stream
  that never ran a GEMM (the library allocates the stream's scratch during
  the capture), then replayed, and the same stream then runs eagerly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import MAX_REL_TOL, MEAN_REL_TOL, bf16_tensor, rel_errors, words_of
from zipserv_asplos26_b200 import runtime

pytestmark = pytest.mark.gpu


def _fp32(w_dev, x):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x.float() @ w_dev.float().t()).to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _case(oracle_mod, m, k, seed):
    w = oracle_mod.llama_weight(m, k, seed=seed)
    return bf16_tensor(w).cuda(), runtime.compress(bf16_tensor(w)).to("cuda")


@pytest.mark.parametrize("m,k,n", [(4096, 4096, 16), (4096, 4096, 128), (4096, 14336, 64),
                                   (4096, 512, 8), (6144, 4096, 1), (1024, 2048, 48)])
def test_last_arrival_route_matches_waiting_reducer(oracle_mod, m, k, n):
    w_dev, packed = _case(oracle_mod, m, k, seed=m + k + n)
    x = torch.randn(n, k, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16).cuda()
    assert runtime.workspace_size(m, n, k)[0] > 0, "shape must split row blocks over CTAs"
    waiting = runtime.linear(x, packed)
    previous = runtime.set_reducer_wait(0)
    try:
        forced = [runtime.linear(x, packed) for _ in range(3)]
    finally:
        runtime.set_reducer_wait(previous)
    again = runtime.linear(x, packed)
    torch.cuda.synchronize()
    assert runtime.device_flags() == 0
    for y in forced + [again]:
        assert torch.equal(y.view(torch.int16), waiting.view(torch.int16))
    mx, mean = rel_errors(words_of(waiting), words_of(_fp32(w_dev, x)))
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)


def test_fused_gemm_while_another_stream_holds_the_sms(oracle_mod):
    w_dev, packed = _case(oracle_mod, 4096, 4096, seed=3)
    g = torch.Generator().manual_seed(4)
    big = (torch.randn(28672, 8192, generator=g) * 0.02).to(torch.bfloat16)
    big_packed = runtime.compress(big).to("cuda")
    del big
    dense = torch.empty(28672, 8192, dtype=torch.bfloat16, device="cuda")
    xs = [torch.randn(n, 4096, generator=g).to(torch.bfloat16).cuda() for n in (16, 64, 128)]
    solo = [runtime.linear(x, packed) for x in xs]
    torch.cuda.synchronize()
    busy, work = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(4):
        outs = []
        with torch.cuda.stream(busy):
            runtime.decompress(big_packed, out=dense)  # persistent grid on every SM
        with torch.cuda.stream(work):
            for x in xs:
                outs.append(runtime.linear(x, packed))
        torch.cuda.synchronize()
        for got, want in zip(outs, solo):
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert runtime.device_flags() == 0


def test_capture_of_an_unseen_shape_on_a_fresh_stream(oracle_mod):
    m, k, n = 1536, 2048, 24
    w_dev, packed = _case(oracle_mod, m, k, seed=21)
    assert runtime.workspace_size(m, n, k)[0] > 0
    x = torch.randn(n, k, generator=torch.Generator().manual_seed(22)).to(torch.bfloat16).cuda()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            y = runtime.linear(x, packed)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        eager = runtime.linear(x, packed)  # the stream's scratch outside the graph
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), eager.view(torch.int16))
    mx, mean = rel_errors(words_of(y), words_of(_fp32(w_dev, x)))
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)
    assert runtime.device_flags() == 0
