"""Runtime knobs (reference: fxpr_vllm/vllm_modules/config.py:5-120).

Environment variables, read once into a frozen process-wide config:

=============================  =======  ==========================================
``VLLM_FXP_FRAC_BITS``          16       fractional bits, 0 <= f < int bits
``VLLM_FXP_INT_BITS``           32       accumulator width: 16, 32 or 64
``VLLM_FXP_NUM_KV_SPLITS``      8        KV splits of the decode attention (>= 1)
``VLLM_FXP_DET_RMSNORM``        on       deterministic RMSNorm
``VLLM_FXP_DET_GEMM``           on       fixed_point_det linear method
``VLLM_FXP_DET_ATTN``           on       CUSTOM attention backend
``VLLM_FXP_DET_LOGPROBS``       on       deterministic sampler log-softmax
=============================  =======  ==========================================

Malformed or out-of-range values log a warning and fall back to the default
(never raise), as in the reference.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass

DEFAULT_FRAC_BITS = 16
DEFAULT_FXP_INT_BITS = 32
DEFAULT_NUM_KV_SPLITS = 8

logger = logging.getLogger("fxpr_vllm")


def _env_int(name: str, default: int) -> int:
    raw = os.getenv(name)
    if raw is None or raw == "":
        return default
    try:
        return int(raw)
    except ValueError:
        logger.warning("Ignoring malformed %s=%r; using default %d", name, raw, default)
        return default


def _env_bool(name: str, default: bool) -> bool:
    raw = os.getenv(name)
    if raw is None or raw == "":
        return default
    return raw.strip().lower() not in ("0", "false", "no", "off")


@dataclass(frozen=True)
class FxpRuntimeConfig:
    frac_bits: int = DEFAULT_FRAC_BITS
    fxp_int_bits: int = DEFAULT_FXP_INT_BITS
    num_kv_splits: int = DEFAULT_NUM_KV_SPLITS
    enable_rmsnorm: bool = True
    enable_gemm: bool = True
    enable_attn: bool = True
    enable_logprobs: bool = True


def load_runtime_config() -> FxpRuntimeConfig:
    """Build a config from the ``VLLM_FXP_*`` environment variables."""
    int_bits = _env_int("VLLM_FXP_INT_BITS", DEFAULT_FXP_INT_BITS)
    if int_bits not in (16, 32, 64):
        logger.warning("Invalid VLLM_FXP_INT_BITS=%d; must be 16/32/64. Using default %d.",
                       int_bits, DEFAULT_FXP_INT_BITS)
        int_bits = DEFAULT_FXP_INT_BITS
    frac_bits = _env_int("VLLM_FXP_FRAC_BITS", DEFAULT_FRAC_BITS)
    if not 0 <= frac_bits < int_bits:
        logger.warning("Invalid VLLM_FXP_FRAC_BITS=%d; must satisfy 0 <= frac_bits < %d. "
                       "Using default %d.", frac_bits, int_bits, DEFAULT_FRAC_BITS)
        frac_bits = DEFAULT_FRAC_BITS
    splits = _env_int("VLLM_FXP_NUM_KV_SPLITS", DEFAULT_NUM_KV_SPLITS)
    if splits < 1:
        logger.warning("Invalid VLLM_FXP_NUM_KV_SPLITS=%d; must be >= 1. Using default %d.",
                       splits, DEFAULT_NUM_KV_SPLITS)
        splits = DEFAULT_NUM_KV_SPLITS
    return FxpRuntimeConfig(
        frac_bits=frac_bits,
        fxp_int_bits=int_bits,
        num_kv_splits=splits,
        enable_rmsnorm=_env_bool("VLLM_FXP_DET_RMSNORM", True),
        enable_gemm=_env_bool("VLLM_FXP_DET_GEMM", True),
        enable_attn=_env_bool("VLLM_FXP_DET_ATTN", True),
        enable_logprobs=_env_bool("VLLM_FXP_DET_LOGPROBS", True),
    )


_runtime_config: FxpRuntimeConfig | None = None


def get_runtime_config() -> FxpRuntimeConfig:
    """Process-wide config, loaded from the environment on first use."""
    global _runtime_config
    if _runtime_config is None:
        _runtime_config = load_runtime_config()
    return _runtime_config


def set_runtime_config(cfg: FxpRuntimeConfig) -> None:
    """Override the process-wide config."""
    global _runtime_config
    _runtime_config = cfg
