"""The vLLM linear method (zipserv_asplos26_b200.vllm_plugin) on CUDA, driven
through the same fake vLLM module tree as the CPU tests: weights loaded on the
host, packed to CUDA after loading, forward through the fused kernel (fixed
and planned dispatch), the large-batch route (bit-exact decode + stock GEMM),
and CUDA-graph capture of the fused route."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from helpers import MAX_REL_TOL, MEAN_REL_TOL, rel_errors, words_of
from test_integration_guards import _State, _fake_vllm, _layer, _vllm_config

pytestmark = pytest.mark.gpu


@pytest.fixture
def fake(monkeypatch, native_lib):
    f = _fake_vllm(monkeypatch)
    monkeypatch.setattr(f.plugin, "_target_device", lambda: torch.device("cuda", 0))
    _State.config = _vllm_config(max_tokens=512)
    yield f
    _State.config = None


def _reference(x, weight, bias):
    """FP32 GEMM rounded to BF16, then the bias added in BF16: the linear
    method's semantics (the reference plugin adds the bias to the BF16 GEMM
    output the same way)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x.float() @ weight.float().T).to(torch.bfloat16) + bias
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_fixed_dispatch_forward(fake):
    method = fake.plugin.ZipServLinearMethod()
    layer, weight = _layer(fake, method, m=512, k=1024)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed and layer.zipserv_sm.is_cuda
    w = weight.cuda()
    bias = torch.randn(512, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    for n in (1, 16, 100):
        x = torch.randn(n, 1024, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16).cuda()
        y = method.apply(layer, x, bias)
        torch.cuda.synchronize()
        mx, mean = rel_errors(words_of(y), words_of(_reference(x, w, bias)))
        assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (n, mx, mean)


def test_planned_dispatch_routes(fake):
    settings = fake.plugin.DispatchSettings(mode="shape", large_batch_tokens=64)
    method = fake.plugin.ZipServLinearMethod(1, settings)
    layer, weight = _layer(fake, method, m=512, k=1024)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed
    w = weight.cuda()
    bias = torch.randn(512, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(5)
    small = torch.randn(32, 1024, generator=g).to(torch.bfloat16).cuda()   # fused route
    large = torch.randn(200, 1024, generator=g).to(torch.bfloat16).cuda()  # decode + stock GEMM
    y = method.apply(layer, small, bias)
    torch.cuda.synchronize()
    mx, mean = rel_errors(words_of(y), words_of(_reference(small, w, bias)))
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)
    # The large batch decodes the weight bit-exactly and runs the same stock
    # GEMM as on the original weight: identical words.
    assert torch.equal(method.apply(layer, large, bias).view(torch.int16),
                       F.linear(large, w, bias).view(torch.int16))


def test_fused_route_in_cuda_graph(fake):
    method = fake.plugin.ZipServLinearMethod()
    layer, weight = _layer(fake, method, m=256, k=512)
    method.process_weights_after_loading(layer)
    x = torch.randn(8, 512, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).cuda()
    eager = method.apply(layer, x)  # also sizes the library's per-stream scratch
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        method.apply(layer, x)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = method.apply(layer, x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16))


def test_padded_rows_forward(fake):
    """pad_rows: a 1000-row layer is packed as 1024 rows (the pad repeats the
    first rows); both routes return exactly the 1000 real output columns."""
    settings = fake.plugin.DispatchSettings(mode="shape", large_batch_tokens=64)
    method = fake.plugin.ZipServLinearMethod(1, settings, pad_rows=True)
    layer, weight = _layer(fake, method, m=1000, k=512)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed and layer.zipserv_metadata[:2] == (1024, 512)
    w = weight.cuda()
    bias = torch.randn(1000, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(9)
    small = torch.randn(16, 512, generator=g).to(torch.bfloat16).cuda()   # fused route
    large = torch.randn(200, 512, generator=g).to(torch.bfloat16).cuda()  # decode + stock GEMM
    y = method.apply(layer, small, bias)
    torch.cuda.synchronize()
    assert y.shape == (16, 1000) and y.is_contiguous()
    mx, mean = rel_errors(words_of(y), words_of(_reference(small, w, bias)))
    assert mx <= MAX_REL_TOL and mean <= MEAN_REL_TOL, (mx, mean)
    assert torch.equal(method.apply(layer, large, bias).view(torch.int16),
                       F.linear(large, w, bias).view(torch.int16))
