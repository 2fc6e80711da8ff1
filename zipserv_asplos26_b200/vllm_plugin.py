"""vLLM quantization method for losslessly compressed BF16 linears, on the
B200 library.

Drop-in for ``zipserv_vllm.vllm_plugin`` (integrations/vllm/zipserv_vllm/
vllm_plugin.py:43-259): the same config name ("zipserv"), config keys,
class names and caller semantics — dense fallback with a logged reason,
online packing of TP-sharded BF16 weights after loading, bias add, optional
planned dispatch with a decode + stock GEMM route for large batches. The
packed weight lives in seven registered CUDA byte buffers and the forward
pass is the ``zipserv_vllm::linear`` custom op of this package's runtime.
"""
from __future__ import annotations

import logging
from typing import Any

import torch
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
_DISPATCH_KEYS = ("large_batch_tokens", "workspace_bytes", "partial_dtype",
                  "decode_workspace_bytes")


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
        # Anything but BF16 activations would need a lossy conversion.
        return [torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # this library is built for sm_100a

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []  # packing is online; the checkpoint stays raw BF16

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "ZipServConfig":
        if config.get("quant_method", "zipserv") != "zipserv":
            raise ValueError("ZipServ expects raw BF16 weights, not another quantization format")
        if config.get("checkpoint_format", "bf16") != "bf16":
            raise ValueError("ZipServ loads raw BF16 checkpoints only")
        ignore = config.get("ignore", [])
        if not isinstance(ignore, list) or any(not isinstance(n, str) for n in ignore):
            raise ValueError("ignore must be a list of exact vLLM module prefixes")
        knobs = {key: config[key] for key in _DISPATCH_KEYS if key in config}
        dispatch = DispatchSettings(mode=config.get("dispatch", "fixed"), **knobs)
        return cls(config.get("split_k", 1), tuple(ignore), dispatch,
                   config.get("pad_rows", False))

    def get_quant_method(self, layer: nn.Module, prefix: str) -> LinearMethodBase | None:
        """Compress dense linears; router gates and ignored prefixes stay stock."""
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


def _keep_dense(layer: nn.Module, weight: Tensor, device: torch.device, reason: str) -> None:
    layer.zipserv_fallback_reason = reason
    layer.zipserv_compressed = False
    layer.weight.data = weight.to(device)


@register_weight_loader_v2_supported_method
class ZipServLinearMethod(LinearMethodBase):
    """Loads TP-sharded BF16 weights on the CPU, packs them after loading and
    replaces each eligible weight by seven CUDA byte buffers."""

    requires_device_loading = False

    def __init__(self, split_k: int = 1, dispatch: DispatchSettings = DEFAULT_DISPATCH,
                 pad_rows: bool = False) -> None:
        self.split_k, self.dispatch, self.pad_rows = split_k, dispatch, pad_rows

    def create_weights(self, layer: nn.Module, input_size_per_partition: int,
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **attrs: Any) -> None:
        if params_dtype != torch.bfloat16:
            raise ValueError("ZipServ requires BF16 checkpoint loading; select --dtype bfloat16")
        stock_loader = attrs.pop("weight_loader")

        def load_bf16(param: nn.Parameter, loaded: Tensor, *args: Any, **kwargs: Any) -> None:
            if loaded.dtype != torch.bfloat16:
                raise ValueError("ZipServ requires BF16 source linear weights; "
                                 "implicit dtype casts are rejected")
            stock_loader(param, loaded, *args, **kwargs)

        weight = ModelWeightParameter(
            data=torch.empty((sum(output_partition_sizes), input_size_per_partition),
                             dtype=params_dtype, device="cpu"),
            input_dim=1, output_dim=0, weight_loader=load_bf16)
        layer.register_parameter("weight", weight)
        set_weight_attrs(weight, attrs)

    def _planned_tokens(self) -> tuple[int | None, Any]:
        from vllm.config import get_current_vllm_config

        config = get_current_vllm_config()
        max_tokens = getattr(config.scheduler_config, "max_num_batched_tokens", None)
        compilation = getattr(config, "compilation_config", None)
        # CUDA-graph padding may exceed the scheduler budget: plan for both.
        graph_max = getattr(compilation, "max_cudagraph_capture_size", None)
        if type(max_tokens) is int and type(graph_max) is int:
            max_tokens = max(max_tokens, graph_max)
        return max_tokens, compilation

    def process_weights_after_loading(self, layer: nn.Module) -> None:
        original = weight = layer.weight.detach()
        rows, k = weight.shape
        layer.zipserv_rows = rows
        # With pad_rows, an output size that is not a multiple of 64 is packed
        # with its first rows repeated up to the next multiple (repeating real
        # rows keeps the pad's exponents inside the matrix's window, where
        # zero rows could make a tile of exceptions that raises the payload
        # capacity of every tile); outputs are cropped back to `rows`.
        if self.pad_rows and rows > 0 and rows % 64:
            extra = -rows % 64
            weight = torch.cat((weight, weight[torch.arange(extra) % rows]), dim=0)
        m = weight.shape[0]
        device = _target_device()
        max_tokens, compilation = self._planned_tokens()
        settings = self.dispatch
        if settings.mode == "fixed":
            reason = startup_rejection(m, k, self.split_k, max_tokens)
        else:
            graph_mode = getattr(getattr(compilation, "cudagraph_mode", None), "name", None)
            if (compilation is None or int(compilation.mode) != 0
                    or graph_mode not in ("NONE", "FULL_DECODE_ONLY")):
                raise ValueError("Planned BF16 dispatch requires compilation mode 0 and eager "
                                 "or full-decode-only CUDA graphs")
            fused_max = (min(max_tokens, settings.large_batch_tokens)
                         if type(max_tokens) is int else None)
            reason = startup_rejection(m, k, 1, fused_max) or decode_budget_rejection(
                m, k, settings)
            graph_max = getattr(compilation, "max_cudagraph_capture_size", None)
            if reason is None and graph_mode == "FULL_DECODE_ONLY" and (
                    type(graph_max) is not int or not 1 <= graph_max <= settings.large_batch_tokens):
                reason = ("Decode graph capture maximum must be positive and within the fused "
                          "token threshold")
            if reason is None:
                from vllm.model_executor.layers.linear import dispatch_unquantized_gemm

                layer.zipserv_stock_gemm = dispatch_unquantized_gemm()
                layer.zipserv_sm_count = torch.cuda.get_device_properties(
                    device).multi_processor_count
        layer.zipserv_max_tokens = max_tokens
        layer.zipserv_fallback_reason = reason
        if reason is not None:
            logger.warning("ZipServ keeps dense weight %s (max_planned_tokens=%s, Split-K=%s): %s",
                           (m, k), max_tokens, self.split_k, reason)
            _keep_dense(layer, original, device, reason)
            return
        if settings.partial_dtype == "fp32":
            require_fp32_partials()
        packed = compress(weight.cpu())
        if packed.storage_bytes >= original.numel() * original.element_size():
            logger.info("ZipServ keeps dense weight %s: packed weight does not shrink", (rows, k))
            _keep_dense(layer, original, device, "Packed weight does not shrink")
            return
        packed = packed.to(device)
        for name, buffer in zip(BUFFER_NAMES, packed.buffers, strict=True):
            layer.register_buffer("zipserv_" + name, buffer)
        layer.zipserv_metadata = (m, k, packed.max_common, packed.max_rare, packed.start_exp)
        layer.zipserv_storage_bytes = packed.storage_bytes
        layer.zipserv_compressed = True
        layer.register_parameter("weight", None)
        if settings.mode != "fixed":
            logger.warning("ZipServ %s dispatch for %s: fused through %s tokens, larger batches "
                           "decode the weight (%s bytes) and use stock GEMM outside graph capture",
                           settings.mode, (m, k), settings.large_batch_tokens, m * k * 2)

    def apply(self, layer: nn.Module, x: Tensor, bias: Tensor | None = None) -> Tensor:
        if not layer.zipserv_compressed:
            return torch.nn.functional.linear(x, layer.weight, bias)
        buffers = [getattr(layer, "zipserv_" + name) for name in BUFFER_NAMES]
        m, k, *_ = layer.zipserv_metadata
        rows = getattr(layer, "zipserv_rows", m)
        settings = self.dispatch
        split = (self.split_k if settings.mode == "fixed" else
                 select_split(m, x.numel() // k, k, layer.zipserv_sm_count, settings,
                              self.split_k))
        if split is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("The large-batch decode route is excluded from CUDA graphs")
            packed = PackedWeight(tuple(buffers), *layer.zipserv_metadata)
            dense = decompress(packed, max_bytes=settings.decode_workspace_bytes)
            return layer.zipserv_stock_gemm(layer, x, dense[:rows], bias)
        y = _linear(x, buffers, *layer.zipserv_metadata, split, settings.partial_dtype == "fp32")
        if rows != m:
            y = y[..., :rows].contiguous()
        return y if bias is None else y + bias
