"""vLLM quantization method for losslessly compressed BF16 linears, on the
B200 library.

vLLM-facing interface, kept as the reference plugin defines it
(integrations/vllm/zipserv_vllm/vllm_plugin.py:43-259) so deployments switch
by import: quantization config name "zipserv", the config keys (split_k,
ignore, dispatch, large_batch_tokens, workspace_bytes, partial_dtype,
decode_workspace_bytes, per_shape_threshold, quant_method, checkpoint_format), the classes
``ZipServConfig`` / ``ZipServLinearMethod``, BF16-only weight loading on the
host, the seven ``zipserv_<stream>`` buffers and the ``zipserv_*`` layer
attributes, dense fallback with a logged reason, and the forward through the
``zipserv_vllm::linear`` custom op.

How it is organised here: loading decides, once per layer, a *route* — the
object its forward calls (``_DenseRoute``: stock linear on the kept weight;
``_FusedRoute``: the fused kernel with the configured split;
``_PlannedRoute``: per-call split from the planner, and above the fused
token threshold bit-exact decompression + the stock GEMM). The reasons a
layer stays dense come from one admission function over the planner's
rejections. Added here: ``pad_rows`` (pack an output size that is not a
multiple of 64 by repeating its first rows, crop outputs).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from vllm.model_executor.layers.linear import (
    LinearBase,
    LinearMethodBase,
    UnquantizedLinearMethod,
    register_weight_loader_v2_supported_method,
)
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
from vllm.model_executor.parameter import ModelWeightParameter
from vllm.model_executor.utils import set_weight_attrs

from .bf16_policy import (
    DispatchSettings,
    decode_budget_rejection,
    fused_token_limit,
    select_split,
    startup_rejection,
)
from .runtime import (
    BUFFER_NAMES,
    PackedWeight,
    _linear,
    compress,
    decompress,
    require_fp32_partials,
)

logger = logging.getLogger(__name__)
DEFAULT_DISPATCH = DispatchSettings()
# Config keys forwarded to DispatchSettings (the planner validates them).
_DISPATCH_KNOBS = ("large_batch_tokens", "workspace_bytes", "partial_dtype",
                   "decode_workspace_bytes", "per_shape_threshold")
_PLANNED_GRAPH_MODES = ("NONE", "FULL_DECODE_ONLY")


@register_quantization_config("zipserv")
class ZipServConfig(QuantizationConfig):
    """Online lossless packing of raw BF16 checkpoints (method "zipserv")."""

    def __init__(self, split_k: int = 1, ignore: tuple[str, ...] = (),
                 dispatch: DispatchSettings = DEFAULT_DISPATCH, pad_rows: bool = False) -> None:
        super().__init__()
        if type(split_k) is not int or split_k < 1:
            raise ValueError("split_k must be positive")
        if type(pad_rows) is not bool:
            raise ValueError("pad_rows must be true or false")
        self.split_k, self.ignore, self.dispatch = split_k, tuple(ignore), dispatch
        self.pad_rows = pad_rows

    def get_name(self) -> str:
        return "zipserv"

    def get_supported_act_dtypes(self) -> list[torch.dtype]:
        return [torch.bfloat16]  # any other activation type would need a lossy cast

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # kernels are built for sm_100a only

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []  # packing happens at load; the checkpoint stays raw BF16

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "ZipServConfig":
        requirements = (
            (config.get("quant_method", "zipserv") == "zipserv",
             "ZipServ expects raw BF16 weights, not another quantization format"),
            (config.get("checkpoint_format", "bf16") == "bf16",
             "ZipServ loads raw BF16 checkpoints only"),
        )
        for ok, message in requirements:
            if not ok:
                raise ValueError(message)
        ignore = config.get("ignore", [])
        if not (isinstance(ignore, list) and all(isinstance(p, str) for p in ignore)):
            raise ValueError("ignore must be a list of exact vLLM module prefixes")
        dispatch = DispatchSettings(mode=config.get("dispatch", "fixed"),
                                    **{key: config[key] for key in _DISPATCH_KNOBS
                                       if key in config})
        return cls(config.get("split_k", 1), tuple(ignore), dispatch,
                   config.get("pad_rows", False))

    def get_quant_method(self, layer: nn.Module, prefix: str) -> LinearMethodBase | None:
        """Dense linears are compressed; router gates and ignored prefixes
        keep vLLM's stock method; other modules are not linears."""
        if not isinstance(layer, LinearBase):
            return None
        from vllm.model_executor.layers.fused_moe.router.gate_linear import GateLinear

        if isinstance(layer, GateLinear) or prefix in self.ignore:
            logger.info("ZipServ keeps stock linear dispatch for %s", prefix)
            return UnquantizedLinearMethod()
        return ZipServLinearMethod(self.split_k, self.dispatch, self.pad_rows)


def _target_device() -> torch.device:
    """The CUDA device packed buffers (or a kept dense weight) move to."""
    return torch.device("cuda", torch.cuda.current_device())


class _Bf16OnlyLoader:
    """Weight loader that refuses anything but BF16 tensors, then defers to
    vLLM's shard loader (a cast would make the packing lossy)."""

    def __init__(self, stock) -> None:
        self.stock = stock

    def __call__(self, param: nn.Parameter, loaded: Tensor, *args: Any, **kwargs: Any) -> None:
        if loaded.dtype != torch.bfloat16:
            raise ValueError("ZipServ requires BF16 source linear weights; "
                             "implicit dtype casts are rejected")
        self.stock(param, loaded, *args, **kwargs)


@dataclass(frozen=True)
class _Budget:
    """What vLLM will run through a layer: the planned maximum batch (the
    scheduler budget or the largest CUDA-graph capture, whichever is larger)
    and the compilation settings planned dispatch depends on."""

    max_tokens: int | None
    graph_mode: str | None
    graph_max: int | None
    compile_mode: int | None

    @classmethod
    def current(cls) -> "_Budget":
        from vllm.config import get_current_vllm_config

        config = get_current_vllm_config()
        tokens = getattr(config.scheduler_config, "max_num_batched_tokens", None)
        comp = getattr(config, "compilation_config", None)
        graph_max = getattr(comp, "max_cudagraph_capture_size", None)
        if type(tokens) is int and type(graph_max) is int:
            tokens = max(tokens, graph_max)
        mode = getattr(getattr(comp, "cudagraph_mode", None), "name", None)
        return cls(tokens, mode, graph_max, None if comp is None else int(comp.mode))


def _admission(m: int, k: int, split_k: int, settings: DispatchSettings,
               budget: _Budget) -> str | None:
    """Why a packed m x k weight must stay dense, or None. Raises for planned
    dispatch under compilation settings it cannot serve."""
    if settings.mode == "fixed":
        return startup_rejection(m, k, split_k, budget.max_tokens)
    if budget.compile_mode != 0 or budget.graph_mode not in _PLANNED_GRAPH_MODES:
        raise ValueError("Planned BF16 dispatch requires compilation mode 0 and eager or "
                         "full-decode-only CUDA graphs")
    limit = fused_token_limit(m, k, settings)
    fused_max = min(budget.max_tokens, limit) if type(budget.max_tokens) is int else None
    reason = (startup_rejection(m, k, 1, fused_max)
              or decode_budget_rejection(m, k, settings))
    if reason is None and budget.graph_mode == "FULL_DECODE_ONLY" and not (
            type(budget.graph_max) is int and 1 <= budget.graph_max <= limit):
        # The decode route cannot be captured, so every captured size must
        # stay on the fused route.
        reason = ("Decode graph capture maximum must be positive and within the fused token "
                  "threshold")
    return reason


# --------------------------------------------------------------- routes
class _DenseRoute:
    """The weight stays a dense parameter; forward is the stock linear."""

    compressed = False

    def __call__(self, layer: nn.Module, x: Tensor, bias: Tensor | None) -> Tensor:
        return F.linear(x, layer.weight, bias)


class _FusedRoute:
    """Fused decompress-GEMM with a fixed split; outputs cropped to the
    layer's real rows when the packed weight was padded."""

    compressed = True

    def __init__(self, rows: int, split_k: int, fp32: bool) -> None:
        self.rows, self.split_k, self.fp32 = rows, split_k, fp32

    @staticmethod
    def buffers(layer: nn.Module) -> list[Tensor]:
        return [getattr(layer, "zipserv_" + name) for name in BUFFER_NAMES]

    def fused(self, layer: nn.Module, x: Tensor, split: int, bias: Tensor | None) -> Tensor:
        y = _linear(x, self.buffers(layer), *layer.zipserv_metadata, split, self.fp32)
        if y.shape[-1] != self.rows:
            y = y[..., :self.rows].contiguous()
        return y if bias is None else y + bias

    def __call__(self, layer: nn.Module, x: Tensor, bias: Tensor | None) -> Tensor:
        return self.fused(layer, x, self.split_k, bias)


class _PlannedRoute(_FusedRoute):
    """Per-call split from the planner; batches above the fused threshold
    decode the weight bit-exactly and run vLLM's stock GEMM (eager only)."""

    def __init__(self, rows: int, split_k: int, fp32: bool, settings: DispatchSettings,
                 sms: int, stock_gemm) -> None:
        super().__init__(rows, split_k, fp32)
        self.settings, self.sms, self.stock_gemm = settings, sms, stock_gemm

    def __call__(self, layer: nn.Module, x: Tensor, bias: Tensor | None) -> Tensor:
        m, k = layer.zipserv_metadata[:2]
        split = select_split(m, x.numel() // k, k, self.sms, self.settings, self.split_k)
        if split is not None:
            return self.fused(layer, x, split, bias)
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("The large-batch decode route is excluded from CUDA graphs")
        packed = PackedWeight(tuple(self.buffers(layer)), *layer.zipserv_metadata)
        dense = decompress(packed, max_bytes=self.settings.decode_workspace_bytes)
        return self.stock_gemm(layer, x, dense[:self.rows], bias)


def _pad_to_tiles(weight: Tensor) -> Tensor:
    """Append copies of the first rows up to the next multiple of 64 rows.
    Repeated real rows keep the pad's exponents inside the matrix's 7-value
    window; zero rows could form a tile of exceptions that would raise the
    payload capacity of every tile."""
    rows = weight.shape[0]
    extra = -rows % 64
    return torch.cat((weight, weight[torch.arange(extra) % rows]), dim=0) if extra else weight


@register_weight_loader_v2_supported_method
class ZipServLinearMethod(LinearMethodBase):
    """BF16 weights load into host memory (TP-sharded by vLLM's loaders);
    after loading each eligible weight is packed and replaced by seven CUDA
    byte buffers, and the layer gets its forward route."""

    requires_device_loading = False

    def __init__(self, split_k: int = 1, dispatch: DispatchSettings = DEFAULT_DISPATCH,
                 pad_rows: bool = False) -> None:
        self.split_k, self.dispatch, self.pad_rows = split_k, dispatch, pad_rows

    def create_weights(self, layer: nn.Module, input_size_per_partition: int,
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **attrs: Any) -> None:
        if params_dtype != torch.bfloat16:
            raise ValueError("ZipServ requires BF16 checkpoint loading; select --dtype bfloat16")
        loader = _Bf16OnlyLoader(attrs.pop("weight_loader"))
        shape = (sum(output_partition_sizes), input_size_per_partition)
        weight = ModelWeightParameter(data=torch.empty(shape, dtype=params_dtype, device="cpu"),
                                      input_dim=1, output_dim=0, weight_loader=loader)
        layer.register_parameter("weight", weight)
        set_weight_attrs(weight, attrs)

    def _keep_dense(self, layer: nn.Module, weight: Tensor, device: torch.device,
                    reason: str) -> None:
        layer.zipserv_fallback_reason = reason
        layer.zipserv_compressed = False
        layer.zipserv_route = _DenseRoute()
        layer.weight.data = weight.to(device)

    def process_weights_after_loading(self, layer: nn.Module) -> None:
        original = layer.weight.detach()
        rows, k = original.shape
        layer.zipserv_rows = rows
        weight = _pad_to_tiles(original) if self.pad_rows and rows > 0 else original
        m = weight.shape[0]
        device = _target_device()
        budget = _Budget.current()
        settings = self.dispatch
        reason = _admission(m, k, self.split_k, settings, budget)
        layer.zipserv_max_tokens = budget.max_tokens
        if reason is not None:
            logger.warning("ZipServ keeps dense weight %s (max_planned_tokens=%s, Split-K=%s): %s",
                           (m, k), budget.max_tokens, self.split_k, reason)
            self._keep_dense(layer, original, device, reason)
            return
        fp32 = settings.partial_dtype == "fp32"
        if fp32:
            require_fp32_partials()
        packed = compress(weight.cpu())
        if packed.storage_bytes >= original.numel() * original.element_size():
            logger.info("ZipServ keeps dense weight %s: packed weight does not shrink", (rows, k))
            self._keep_dense(layer, original, device, "Packed weight does not shrink")
            return
        packed = packed.to(device)  # one copy of the packed arena
        for name, buffer in zip(BUFFER_NAMES, packed.buffers, strict=True):
            layer.register_buffer("zipserv_" + name, buffer)
        layer.zipserv_metadata = (m, k, packed.max_common, packed.max_rare, packed.start_exp)
        layer.zipserv_storage_bytes = packed.storage_bytes
        layer.zipserv_fallback_reason = None
        layer.zipserv_compressed = True
        layer.register_parameter("weight", None)
        if settings.mode == "fixed":
            layer.zipserv_route = _FusedRoute(rows, self.split_k, fp32)
            return
        from vllm.model_executor.layers.linear import dispatch_unquantized_gemm

        layer.zipserv_stock_gemm = dispatch_unquantized_gemm()
        layer.zipserv_sm_count = torch.cuda.get_device_properties(device).multi_processor_count
        layer.zipserv_route = _PlannedRoute(rows, self.split_k, fp32, settings,
                                            layer.zipserv_sm_count, layer.zipserv_stock_gemm)
        logger.warning("ZipServ %s dispatch for %s: fused through %s tokens, larger batches "
                       "decode the weight (%s bytes) and use stock GEMM outside graph capture",
                       settings.mode, (m, k), fused_token_limit(m, k, settings), m * k * 2)

    def apply(self, layer: nn.Module, x: Tensor, bias: Tensor | None = None) -> Tensor:
        route = getattr(layer, "zipserv_route", None)
        if route is None:  # a layer whose weights were never processed
            route = _FusedRoute(layer.zipserv_rows, self.split_k, False) \
                if getattr(layer, "zipserv_compressed", False) else _DenseRoute()
        return route(layer, x, bias)
