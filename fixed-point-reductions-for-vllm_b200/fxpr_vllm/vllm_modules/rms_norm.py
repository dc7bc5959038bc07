"""Deterministic RMSNorm layer (reference: fxpr_vllm/vllm_modules/rms_norm.py:11-99).

``forward_cuda`` runs one fused kernel on the activation dtype (bf16 in and
out; the reference's fp32 up/down-casts give the same bits and are skipped).
``forward_native`` is the path vLLM takes when custom ops are compiled out:
it calls the same CUDA op (a torch.library op, traceable) -- there is no CPU
implementation; CPU tensors raise.
"""

from __future__ import annotations

import torch
from vllm.model_executor.custom_op import CustomOp
from vllm.model_executor.layers.layernorm import RMSNorm

from .. import library_ops  # noqa: F401
from .config import get_runtime_config


@CustomOp.register("rms_norm")
@CustomOp.register_oot(name="RMSNorm")
class DeterministicRMSNorm(RMSNorm):
    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        cfg = get_runtime_config()
        self._fxp_frac_bits = cfg.frac_bits
        self._fxp_int_bits = cfg.fxp_int_bits

    def forward_cuda(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if not x.is_cuda:
            raise RuntimeError("DeterministicRMSNorm requires CUDA tensors (no CPU implementation)")
        if residual is not None:
            # residual += x in place, as vLLM's own fused add + RMSNorm does
            # (the reference returns an updated copy; callers use the returned one)
            out = torch.ops.fxpr.rms_norm_fxp_residual(
                x, residual, self.weight, self.variance_epsilon, self._fxp_frac_bits,
                self._fxp_int_bits)
            return out, residual
        return torch.ops.fxpr.rms_norm_fxp(x, self.weight, self.variance_epsilon,
                                           self._fxp_frac_bits, self._fxp_int_bits)

    def forward_native(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        return self.forward_cuda(x, residual)
