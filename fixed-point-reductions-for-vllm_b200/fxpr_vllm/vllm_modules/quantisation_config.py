"""``fixed_point_det`` quantisation method: every linear layer runs the
fixed-point GEMM (reference: fxpr_vllm/vllm_modules/quantisation_config.py:25-187).

Differences from the reference that do not change results:

* the weight stays in vLLM's ``[N, K]`` layout (bf16); the GEMM reads the
  transposed view K-contiguously instead of a transposed copy;
* row-parallel layers under TP > 1 reduce their *integer* partials
  (``tp_allreduce.integer_all_reduce``) before X2F + bias, with the bias added
  on every rank after the reduce, so outputs are identical for every TP degree
  (the reference float-allreduces after X2F, which is not TP-invariant).

Addition (not in the reference, whose ``get_quant_method`` returns ``None``
for the LM head, quantisation_config.py:91-93): with ``VLLM_FXP_DET_LM_HEAD``
on (the default) the ``ParallelLMHead`` logits GEMM is fixed-point too
(:class:`FixedPointLMHeadMethod`), so no float reduction is left between the
last hidden state and the greedy argmax. Vocab-parallel shards are gathered,
not summed, so the logits stay independent of the TP degree.
"""

from __future__ import annotations

import logging
from collections.abc import Sequence
from typing import Any

import torch
import torch.nn as nn
from vllm.model_executor.layers.linear import LinearBase, RowParallelLinear
from vllm.model_executor.layers.vocab_parallel_embedding import (
    ParallelLMHead,
    UnquantizedEmbeddingMethod,
)
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import (
    QuantizationConfig,
    QuantizeMethodBase,
)
from vllm.model_executor.parameter import ModelWeightParameter

from .. import library_ops  # noqa: F401  (registers torch.ops.fxpr.*)
from ..fixed_point_kernels.fixed_point import fixed_tl_dtype, int_bits_of
from .config import DEFAULT_FRAC_BITS, get_runtime_config
from .tp_allreduce import integer_all_reduce_op  # noqa: F401  (registers fxpr::integer_all_reduce)

logger = logging.getLogger("fxpr_vllm")


@register_quantization_config("fixed_point_det")
class FixedPointConfig(QuantizationConfig):
    def __init__(self, frac_bits: int = DEFAULT_FRAC_BITS) -> None:
        super().__init__()
        int_bits = int_bits_of(fixed_tl_dtype(get_runtime_config().fxp_int_bits))
        if not isinstance(frac_bits, int) or not 0 <= frac_bits < int_bits:
            raise ValueError(f"frac_bits must be an int in [0, {int_bits}); got {frac_bits!r}")
        self.frac_bits = frac_bits

    def __repr__(self) -> str:
        return f"FixedPointConfig(frac_bits={self.frac_bits})"

    @classmethod
    def get_name(cls) -> str:
        return "fixed_point_det"

    @classmethod
    def get_supported_act_dtypes(cls) -> list[torch.dtype]:
        return [torch.float16, torch.bfloat16, torch.float32]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels

    @classmethod
    def get_config_filenames(cls) -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "FixedPointConfig":
        return cls(frac_bits=config.get("frac_bits", get_runtime_config().frac_bits))

    def get_quant_method(self, layer: nn.Module, prefix: str) -> "QuantizeMethodBase | None":
        if isinstance(layer, LinearBase):
            return FixedPointLinearMethod(self)
        if isinstance(layer, ParallelLMHead) and get_runtime_config().enable_lm_head:
            return FixedPointLMHeadMethod(self)
        return None

    def get_scaled_act_names(self) -> list[str]:
        return []


class FixedPointLinearMethod(QuantizeMethodBase):
    def __init__(self, config: FixedPointConfig) -> None:
        self.config = config
        self.fxp_int_bits = get_runtime_config().fxp_int_bits

    def create_weights(self, layer: nn.Module, input_size_per_partition: int,
                       output_partition_sizes: Sequence[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **extra_weight_attrs: Any) -> None:
        weight = ModelWeightParameter(
            data=torch.empty(sum(output_partition_sizes), input_size_per_partition,
                             dtype=params_dtype),
            input_dim=1,
            output_dim=0,
            weight_loader=extra_weight_attrs.get("weight_loader"),
        )
        layer.register_parameter("weight", weight)

    def process_weights_after_loading(self, layer: nn.Module) -> None:
        """Keep the weight as bf16 ``[N, K]``; expose ``weight_t`` = its ``[K, N]``
        view. Row-parallel layers under TP > 1 switch to the integer reduce."""
        with torch.no_grad():
            w = layer.weight.data
            if w.dtype != torch.bfloat16:
                w = w.to(torch.bfloat16)
            w = w.contiguous()
        del layer.weight
        layer.register_parameter("weight", None)
        layer.fxp_weight = w
        layer.weight_t = w.t()
        layer.fxp_int_reduce = False
        if isinstance(layer, RowParallelLinear) and getattr(layer, "tp_size", 1) > 1 \
                and layer.reduce_results:
            layer.reduce_results = False  # the float allreduce is replaced
            layer.fxp_int_reduce = True

    def apply(self, layer: nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        orig_dtype = x.dtype
        w_t = layer.weight_t
        x2d = x.reshape(-1, x.shape[-1])
        if x2d.dtype != w_t.dtype:
            x2d = x2d.to(w_t.dtype)  # quantisation_config.py:176-177
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        acc = torch.ops.fxpr.gemm_fxp_int(x2d, w_t, self.config.frac_bits, self.fxp_int_bits)
        if getattr(layer, "fxp_int_reduce", False):
            acc = torch.ops.fxpr.integer_all_reduce(acc)
            # bias after the reduce on every rank (vLLM passes it to rank 0 only)
            if layer.bias is not None and not layer.skip_bias_add:
                bias = layer.bias
        out = torch.ops.fxpr.fixed_to_float_bias(acc, bias, self.config.frac_bits,
                                                 self.fxp_int_bits, orig_dtype)
        return out.view(*x.shape[:-1], out.shape[-1])


class FixedPointLMHeadMethod(UnquantizedEmbeddingMethod):
    """Logits of a ``ParallelLMHead`` through the fixed-point GEMM: the weight
    stays the bf16 ``[vocab_shard, hidden]`` parameter (possibly tied to the
    input embedding, whose lookup is unchanged), ``x`` is cast to the weight
    dtype, and each rank computes its vocabulary shard as
    ``cast(X2F(sum_k F2X(x * w)) + bias)``, like FixedPointLinearMethod.apply."""

    def __init__(self, config: FixedPointConfig) -> None:
        super().__init__()
        self.config = config
        self.fxp_int_bits = get_runtime_config().fxp_int_bits

    def apply(self, layer: nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        w = layer.weight
        if w.dtype != torch.bfloat16:
            w = w.to(torch.bfloat16)
        x2d = x.reshape(-1, x.shape[-1])
        if x2d.dtype != w.dtype:
            x2d = x2d.to(w.dtype)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        acc = torch.ops.fxpr.gemm_fxp_int(x2d, w.t(), self.config.frac_bits, self.fxp_int_bits)
        out = torch.ops.fxpr.fixed_to_float_bias(acc, bias, self.config.frac_bits, self.fxp_int_bits,
                                                 x.dtype)
        return out.view(*x.shape[:-1], out.shape[-1])
