"""Deterministic sampler log-softmax (reference: fxpr_vllm/vllm_modules/sampling.py:8-31)."""

from __future__ import annotations

import torch

from ..fixed_point_kernels.softmax import log_softmax_fxp
from .config import get_runtime_config


def deterministic_log_softmax(logits: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Log-softmax with a fixed-point exp-sum; bitwise reproducible."""
    assert logits.is_cuda, "Input tensor must be on CUDA device"
    cfg = get_runtime_config()
    return log_softmax_fxp(logits, fxp_dtype=cfg.fxp_int_bits, dim=dim, frac_bits=cfg.frac_bits)
