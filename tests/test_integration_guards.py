"""Planner limits and the vLLM linear method on a fake vLLM module tree
(reference tests/test_integration_guards.py:77-377): CPU only.

The fake tree provides exactly the vLLM names the plugin imports, with stub
classes, so the plugin's caller semantics (config parsing, which layers are
compressed, weight creation and loading guards, dense fallbacks with their
reasons, buffer registration, dense forward) run without vLLM or a GPU.
"""
from __future__ import annotations

import importlib
import sys
import types
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch import nn

from zipserv_asplos26_b200 import bf16_policy as policy


# --------------------------------------------------------------- planner
def test_gemm_rejection_matches_native_contract(oracle_mod):
    lib = oracle_mod.lib()
    for m, n, k, split in [(64, 1, 64, 1), (64, 0, 64, 1), (64, 8, 256, 4), (64, 8, 256, 3),
                           (96, 8, 64, 1), (64, -1, 64, 1), (64 * 65536, 1, 64, 1),
                           (4096, 1 << 20, 4096, 1), (4096, 16, 4096, 16)]:
        assert (policy.gemm_rejection(m, n, k, split) is None) == bool(
            lib.oracle_valid_gemm(m, n, k, split)), (m, n, k, split)
    assert policy.gemm_rejection(64, 1.0, 64, 1)  # non-integers rejected


def test_startup_and_decode_budget_rejections():
    assert "max_num_batched_tokens" in policy.startup_rejection(64, 64, 1, None)
    assert policy.startup_rejection(4096, 4096, 1, 8192) is None
    assert "int32" in policy.startup_rejection(65536, 65536, 1, 1)
    s = policy.DispatchSettings(mode="shape", decode_workspace_bytes=4096 * 4096 * 2 - 1)
    assert "decode_workspace_bytes" in policy.decode_budget_rejection(4096, 4096, s)
    assert policy.decode_budget_rejection(4096, 4096, policy.DispatchSettings()) is None


def test_per_shape_threshold():
    """With per_shape_threshold each layer is also capped at its
    measured B200 crossover, smaller weights switching to decompression +
    stock GEMM at fewer tokens."""
    limits = [policy.b200_token_limit(m, k) for m, k in
              ((4096, 4096), (6144, 4096), (4096, 14336), (28672, 4096), (57344, 8192))]
    assert limits == sorted(limits) and all(v >= 1 for v in limits)
    on = policy.DispatchSettings(mode="shape", per_shape_threshold=True)
    off = policy.DispatchSettings(mode="shape")
    small, large = (4096, 4096), (28672, 4096)
    n = policy.b200_token_limit(*small) + 1
    assert policy.select_split(*small[:1], n, small[1], 148, on) is None
    assert policy.select_split(*small[:1], n, small[1], 148, off) is not None
    assert policy.fused_token_limit(*large, on) == min(768, policy.b200_token_limit(*large))
    capped = policy.DispatchSettings(mode="shape", per_shape_threshold=True, large_batch_tokens=8)
    assert policy.fused_token_limit(*large, capped) == 8
    with pytest.raises(ValueError):
        policy.DispatchSettings(per_shape_threshold=1)


@pytest.mark.parametrize("bad", [dict(mode="auto"), dict(partial_dtype="fp16"),
                                 dict(large_batch_tokens=0), dict(workspace_bytes=-1),
                                 dict(decode_workspace_bytes=1.5)])
def test_dispatch_settings_validation(bad):
    with pytest.raises(ValueError):
        policy.DispatchSettings(**bad)


def test_split_candidates_and_selection():
    cands = policy.split_candidates(4096, 16, 4096, 148, 64 << 20)
    assert cands and all(64 % c.split_k == 0 and c.workspace_bytes == 0 for c in cands)
    assert max(c.split_k for c in cands) <= policy.MAX_CLUSTER
    shape = policy.DispatchSettings(mode="shape")
    best = policy.select_split(4096, 16, 4096, 148, shape)
    assert best == min(cands, key=lambda c: (c.score, c.split_k)).split_k
    assert best > 1  # 32 row blocks alone leave most of 148 SMs idle
    assert policy.select_split(28672, 16, 4096, 148, shape) == 1  # 224 blocks fill the GPU
    assert policy.select_split(4096, 4096, 4096, 148, shape) is None  # large batch
    tokens = policy.DispatchSettings(mode="tokens")
    assert policy.select_split(4096, 16, 4096, 148, tokens) == 8
    assert policy.select_split(4096, 64, 4096, 148, tokens) == 4
    assert policy.select_split(4096, 16, 4096, 148, policy.DispatchSettings(), 2) == 2
    assert policy.split_candidates(96, 1, 64, 148, 0) == ()
    with pytest.raises(ValueError):
        policy.split_candidates(64, 1, 64, 0, 0)


# ------------------------------------------------------------ fake vLLM
class _State:
    config = None


def _fake_vllm(monkeypatch):
    def module(name, **attrs):
        mod = types.ModuleType(name)
        mod.__dict__.update(attrs)
        monkeypatch.setitem(sys.modules, name, mod)
        return mod

    class LinearBase(nn.Module):
        pass

    class GateLinear(LinearBase):
        pass

    class LinearMethodBase:
        pass

    class UnquantizedLinearMethod(LinearMethodBase):
        pass

    class QuantizationConfig:
        def __init__(self):
            pass

    class ModelWeightParameter(nn.Parameter):
        def __new__(cls, data, input_dim, output_dim, weight_loader):
            p = super().__new__(cls, data, requires_grad=False)
            p.input_dim, p.output_dim, p.weight_loader = input_dim, output_dim, weight_loader
            return p

    def set_weight_attrs(param, attrs):
        for key, value in attrs.items():
            setattr(param, key, value)

    def dispatch_unquantized_gemm():
        return lambda layer, x, weight, bias: F.linear(x, weight, bias)

    registered = {}
    for name in ("vllm", "vllm.model_executor", "vllm.model_executor.layers",
                 "vllm.model_executor.layers.fused_moe",
                 "vllm.model_executor.layers.fused_moe.router"):
        module(name)
    module("vllm.model_executor.layers.linear", LinearBase=LinearBase,
           LinearMethodBase=LinearMethodBase, UnquantizedLinearMethod=UnquantizedLinearMethod,
           register_weight_loader_v2_supported_method=lambda cls: cls,
           dispatch_unquantized_gemm=dispatch_unquantized_gemm)
    module("vllm.model_executor.layers.quantization",
           register_quantization_config=lambda name: (lambda cls: registered.setdefault(name, cls)))
    module("vllm.model_executor.layers.quantization.base_config",
           QuantizationConfig=QuantizationConfig)
    module("vllm.model_executor.parameter", ModelWeightParameter=ModelWeightParameter)
    module("vllm.model_executor.utils", set_weight_attrs=set_weight_attrs)
    module("vllm.config", get_current_vllm_config=lambda: _State.config)
    module("vllm.model_executor.layers.fused_moe.router.gate_linear", GateLinear=GateLinear)
    monkeypatch.delitem(sys.modules, "zipserv_asplos26_b200.vllm_plugin", raising=False)
    plugin = importlib.import_module("zipserv_asplos26_b200.vllm_plugin")
    monkeypatch.setattr(plugin, "_target_device", lambda: torch.device("cpu"))
    return SimpleNamespace(plugin=plugin, LinearBase=LinearBase, GateLinear=GateLinear,
                           Unquantized=UnquantizedLinearMethod, registered=registered)


def _vllm_config(max_tokens=256, mode=0, graph="NONE", graph_max=None):
    return SimpleNamespace(
        scheduler_config=SimpleNamespace(max_num_batched_tokens=max_tokens),
        compilation_config=SimpleNamespace(mode=mode, cudagraph_mode=SimpleNamespace(name=graph),
                                           max_cudagraph_capture_size=graph_max))


@pytest.fixture
def fake(monkeypatch, native_lib):
    f = _fake_vllm(monkeypatch)
    _State.config = _vllm_config()
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda dev: SimpleNamespace(multi_processor_count=148))
    yield f
    _State.config = None


def _layer(fake, method, m=128, k=256, weight=None):
    layer = fake.LinearBase()
    loaded = []
    method.create_weights(layer, k, [m], k, m, torch.bfloat16,
                          weight_loader=lambda p, w: (loaded.append(1), p.data.copy_(w)))
    if weight is None:
        g = torch.Generator().manual_seed(m + k)
        weight = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
    layer.weight.weight_loader(layer.weight, weight)
    assert loaded == [1]
    return layer, weight


def test_config_parsing(fake):
    cfg = fake.plugin.ZipServConfig.from_config(
        {"split_k": 2, "ignore": ["lm_head"], "dispatch": "shape", "large_batch_tokens": 512})
    assert (cfg.split_k, cfg.ignore, cfg.dispatch.mode, cfg.dispatch.large_batch_tokens) == (
        2, ("lm_head",), "shape", 512)
    assert fake.registered["zipserv"] is fake.plugin.ZipServConfig
    assert cfg.get_name() == "zipserv" and cfg.get_supported_act_dtypes() == [torch.bfloat16]
    for bad in ({"quant_method": "fp8"}, {"checkpoint_format": "fp8"}, {"ignore": "lm_head"},
                {"ignore": [1]}, {"split_k": 0}, {"dispatch": "auto"}):
        with pytest.raises(ValueError):
            fake.plugin.ZipServConfig.from_config(bad)


def test_quant_method_selection(fake):
    cfg = fake.plugin.ZipServConfig(split_k=1, ignore=("model.lm_head",))
    assert cfg.get_quant_method(nn.Linear(4, 4), "x") is None
    assert isinstance(cfg.get_quant_method(fake.GateLinear(), "router"), fake.Unquantized)
    assert isinstance(cfg.get_quant_method(fake.LinearBase(), "model.lm_head"), fake.Unquantized)
    method = cfg.get_quant_method(fake.LinearBase(), "model.layers.0.qkv")
    assert isinstance(method, fake.plugin.ZipServLinearMethod) and method.split_k == 1


def test_weight_creation_guards(fake):
    method = fake.plugin.ZipServLinearMethod()
    with pytest.raises(ValueError, match="BF16"):
        method.create_weights(fake.LinearBase(), 64, [64], 64, 64, torch.float16,
                              weight_loader=lambda *a: None)
    layer = fake.LinearBase()
    method.create_weights(layer, 256, [64, 64], 256, 128, torch.bfloat16, weight_loader=lambda *a: None,
                          extra_attr=7)
    assert tuple(layer.weight.shape) == (128, 256) and layer.weight.device.type == "cpu"
    assert layer.weight.extra_attr == 7
    with pytest.raises(ValueError, match="implicit dtype casts"):
        layer.weight.weight_loader(layer.weight, torch.zeros(128, 256))


def test_compressible_weight_is_packed_and_registered(fake):
    method = fake.plugin.ZipServLinearMethod()
    layer, weight = _layer(fake, method)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed and layer.zipserv_fallback_reason is None
    assert layer.weight is None
    from zipserv_asplos26_b200.runtime import BUFFER_NAMES
    bufs = [getattr(layer, "zipserv_" + n) for n in BUFFER_NAMES]
    assert layer.zipserv_storage_bytes == sum(b.numel() for b in bufs) < weight.numel() * 2
    assert layer.zipserv_metadata[:2] == (128, 256)


def test_dense_fallbacks_keep_the_weight_and_run_stock_linear(fake):
    method = fake.plugin.ZipServLinearMethod()
    # Incompressible weight (all 65536 bit patterns): packing would not shrink.
    words = np.random.default_rng(0).integers(0, 65536, size=(128, 256), dtype=np.uint16)
    layer, weight = _layer(fake, method, weight=torch.from_numpy(words.view(np.int16)).view(torch.bfloat16))
    method.process_weights_after_loading(layer)
    assert not layer.zipserv_compressed
    assert layer.zipserv_fallback_reason == "Packed weight does not shrink"
    x = torch.randn(3, 256).to(torch.bfloat16)
    bias = torch.randn(128).to(torch.bfloat16)
    # Same stock computation on both sides: compare bit patterns (NaN-safe).
    assert torch.equal(method.apply(layer, x, bias).view(torch.int16),
                       F.linear(x, weight, bias).view(torch.int16))
    # No planned batch size: the layer stays dense with the planner's reason.
    _State.config = _vllm_config(max_tokens=None)
    layer, _ = _layer(fake, method)
    method.process_weights_after_loading(layer)
    assert not layer.zipserv_compressed and "max_num_batched_tokens" in layer.zipserv_fallback_reason


def test_planned_dispatch_guards(fake):
    shape = fake.plugin.DispatchSettings(mode="shape")
    method = fake.plugin.ZipServLinearMethod(1, shape)
    _State.config = _vllm_config(mode=3)
    with pytest.raises(ValueError, match="compilation mode 0"):
        method.process_weights_after_loading(_layer(fake, method)[0])
    _State.config = _vllm_config(graph="FULL_DECODE_ONLY", graph_max=4096)
    layer, _ = _layer(fake, method)
    method.process_weights_after_loading(layer)
    assert "graph capture maximum" in layer.zipserv_fallback_reason
    small_budget = fake.plugin.ZipServLinearMethod(1, fake.plugin.DispatchSettings(
        mode="shape", decode_workspace_bytes=1024))
    _State.config = _vllm_config()
    layer, _ = _layer(fake, small_budget)
    small_budget.process_weights_after_loading(layer)
    assert "decode_workspace_bytes" in layer.zipserv_fallback_reason
    layer, _ = _layer(fake, method)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed and layer.zipserv_sm_count == 148
    assert layer.zipserv_stock_gemm is not None


def test_unaligned_rows_stay_dense_unless_padding_is_requested(fake, oracle_mod):
    """An output size that is not a multiple of 64 keeps the stock weight by
    default (the reference plugin's behaviour); with `pad_rows` it is packed
    as the next multiple of 64 rows, the pad repeating the first rows."""
    method = fake.plugin.ZipServLinearMethod()
    layer, weight = _layer(fake, method, m=100, k=256)
    method.process_weights_after_loading(layer)
    assert not layer.zipserv_compressed and "64-aligned" in layer.zipserv_fallback_reason
    assert torch.equal(layer.weight.data.view(torch.int16), weight.view(torch.int16))

    cfg = fake.plugin.ZipServConfig.from_config({"pad_rows": True})
    method = cfg.get_quant_method(fake.LinearBase(), "model.layers.0.o_proj")
    assert method.pad_rows
    layer, weight = _layer(fake, method, m=100, k=256)
    method.process_weights_after_loading(layer)
    assert layer.zipserv_compressed and layer.zipserv_rows == 100
    m, k, _, _, start_exp = layer.zipserv_metadata
    assert (m, k) == (128, 256)
    from zipserv_asplos26_b200.runtime import BUFFER_NAMES
    buffers = [getattr(layer, "zipserv_" + n).numpy() for n in BUFFER_NAMES]
    padded = torch.cat((weight, weight[:28])).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle_mod.decode(buffers, m, k, start_exp), padded)
    with pytest.raises(ValueError):
        fake.plugin.ZipServConfig.from_config({"pad_rows": "yes"})
