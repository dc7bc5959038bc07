"""Runtime knobs (reference: fxpr_vllm/vllm_modules/config.py:5-120).

Environment variables, read once into a frozen process-wide config:

=============================  =======  ==========================================
``VLLM_FXP_INT_BITS``           32       accumulator width: 16, 32 or 64
``VLLM_FXP_FRAC_BITS``          16       fractional bits, 0 <= f < int bits
``VLLM_FXP_NUM_KV_SPLITS``      8        KV-split hint of the decode attention (>= 1)
``VLLM_FXP_DET_RMSNORM``        on       deterministic RMSNorm
``VLLM_FXP_DET_GEMM``           on       fixed_point_det linear method
``VLLM_FXP_DET_ATTN``           on       CUSTOM attention backend
``VLLM_FXP_DET_LOGPROBS``       on       deterministic sampler log-softmax
``VLLM_FXP_DET_LM_HEAD``        on       fixed-point LM-head logits GEMM (an addition:
                                         the reference's LM head is a float GEMM)
=============================  =======  ==========================================

A malformed or out-of-range value logs a warning and falls back to the
default; nothing raises. The knobs are described by two tables below and
resolved in table order, so a rule may depend on a knob resolved before it
(the fraction width is checked against the accumulator width).

``VLLM_FXP_NUM_KV_SPLITS`` never changes a result (every split count gives
the same bits). The default decode path balances its work over the SMs by
itself and ignores it; only the scratch-free cluster path reads it, as an
upper bound on the splits per request.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Callable, Mapping

DEFAULT_FRAC_BITS = 16
DEFAULT_FXP_INT_BITS = 32
DEFAULT_NUM_KV_SPLITS = 8

logger = logging.getLogger("fxpr_vllm")


@dataclass(frozen=True)
class _IntKnob:
    """An integer environment knob: its config field, default, and the rule a
    value must meet given the knobs already resolved (``rule`` returns None
    when the value is acceptable, else the text of the rule it breaks)."""

    env: str
    field: str
    default: int
    rule: Callable[[int, Mapping[str, object]], str | None]


_INT_KNOBS = (
    _IntKnob("VLLM_FXP_INT_BITS", "fxp_int_bits", DEFAULT_FXP_INT_BITS,
             lambda v, _: None if v in (16, 32, 64) else "must be 16/32/64"),
    _IntKnob("VLLM_FXP_FRAC_BITS", "frac_bits", DEFAULT_FRAC_BITS,
             lambda v, got: None if 0 <= v < got["fxp_int_bits"]
             else f"must satisfy 0 <= frac_bits < {got['fxp_int_bits']}"),
    _IntKnob("VLLM_FXP_NUM_KV_SPLITS", "num_kv_splits", DEFAULT_NUM_KV_SPLITS,
             lambda v, _: None if v >= 1 else "must be >= 1"),
)

# on/off switches: config field -> environment variable (all default on)
_SWITCHES = {
    "enable_rmsnorm": "VLLM_FXP_DET_RMSNORM",
    "enable_gemm": "VLLM_FXP_DET_GEMM",
    "enable_attn": "VLLM_FXP_DET_ATTN",
    "enable_logprobs": "VLLM_FXP_DET_LOGPROBS",
    "enable_lm_head": "VLLM_FXP_DET_LM_HEAD",
}
_OFF_WORDS = frozenset({"0", "false", "no", "off"})


@dataclass(frozen=True)
class FxpRuntimeConfig:
    frac_bits: int = DEFAULT_FRAC_BITS
    fxp_int_bits: int = DEFAULT_FXP_INT_BITS
    num_kv_splits: int = DEFAULT_NUM_KV_SPLITS
    enable_rmsnorm: bool = True
    enable_gemm: bool = True
    enable_attn: bool = True
    enable_logprobs: bool = True
    enable_lm_head: bool = True


def _resolve_int(knob: _IntKnob, env: Mapping[str, str], got: Mapping[str, object]) -> int:
    text = env.get(knob.env, "")
    if text == "":
        return knob.default
    try:
        value = int(text)
    except ValueError:
        logger.warning("Ignoring malformed %s=%r; using default %d", knob.env, text, knob.default)
        return knob.default
    broken = knob.rule(value, got)
    if broken is not None:
        logger.warning("Invalid %s=%d; %s. Using default %d.", knob.env, value, broken, knob.default)
        return knob.default
    return value


def _resolve_switch(name: str, env: Mapping[str, str]) -> bool:
    text = env.get(name, "")
    return True if text == "" else text.strip().lower() not in _OFF_WORDS


def load_runtime_config(env: Mapping[str, str] | None = None) -> FxpRuntimeConfig:
    """Build a config from the ``VLLM_FXP_*`` variables of ``env`` (default:
    the process environment)."""
    env = os.environ if env is None else env
    got: dict[str, object] = {}
    for knob in _INT_KNOBS:
        got[knob.field] = _resolve_int(knob, env, got)
    for field, name in _SWITCHES.items():
        got[field] = _resolve_switch(name, env)
    return FxpRuntimeConfig(**got)


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
