"""Plugin entry point (reference: fxpr_vllm/register.py:15-117).

``register()`` is vLLM's general-plugin hook (``vllm.general_plugins``:
``fxpr_vllm = fxpr_vllm.register:register``). It is idempotent, gated per
component by the ``VLLM_FXP_DET_*`` knobs and transactional: if a step fails,
the steps already applied are undone and the error is re-raised.
Importing this module registers the ``fixed_point_det`` quantisation method.
"""

from __future__ import annotations

import logging
from typing import Callable

from . import monkey_patches
from .vllm_modules import quantisation_config  # noqa: F401  (registers fixed_point_det)
from .vllm_modules.config import get_runtime_config

logger = logging.getLogger("fxpr_vllm")

_registered = False


def register() -> None:
    """Install the deterministic components into vLLM (safe to call repeatedly)."""
    global _registered
    if _registered:
        return
    _registered = True
    cfg = get_runtime_config()
    logger.info("Runtime Config: frac_bits=%d fxp_int_bits=%d num_kv_splits=%d rmsnorm=%s "
                "gemm=%s attn=%s logprobs=%s", cfg.frac_bits, cfg.fxp_int_bits,
                cfg.num_kv_splits, cfg.enable_rmsnorm, cfg.enable_gemm, cfg.enable_attn,
                cfg.enable_logprobs)
    from . import _native, library_ops  # noqa: F401

    _native.load()  # fail loudly now if the CUDA library is missing
    steps: list[tuple[bool, str, Callable[[], object], Callable[[], None]]] = [
        (cfg.enable_rmsnorm, "RMSNorm", monkey_patches.patch_rms_norm, _undo_rms_norm),
        (cfg.enable_gemm, "GEMM (fixed_point_det)", _noop, _noop),
        (cfg.enable_attn, "Attention", monkey_patches.patch_attention_backend, _undo_attention),
        (cfg.enable_logprobs, "Sampler", monkey_patches.patch_sampler, _undo_sampler),
    ]
    done: list[Callable[[], None]] = []
    name = ""
    try:
        for enabled, name, do, undo in steps:
            if not enabled:
                logger.info("%s registration skipped (disabled)", name)
                continue
            do()
            done.append(undo)
            logger.info("%s registered", name)
    except Exception as e:
        logger.error("Error during %s registration: %s; rolling back", name, e)
        for undo in reversed(done):
            try:
                undo()
            except Exception as undo_err:
                logger.error("Rollback step failed: %s", undo_err)
        _registered = False
        raise


def _noop() -> None:
    """fixed_point_det registers at import time; nothing to do here."""
    return None


def _undo_rms_norm() -> None:
    try:
        import vllm.model_executor.layers.layernorm as layernorm_mod
        from vllm.model_executor.custom_op import op_registry

        op_registry.pop("rms_norm", None)
        base = layernorm_mod.RMSNorm.__mro__[1] if hasattr(layernorm_mod.RMSNorm, "_fxp_frac_bits") else None
        if base is not None:
            layernorm_mod.RMSNorm = base
    except Exception as e:  # pragma: no cover
        logger.warning("RMSNorm rollback failed: %s", e)


def _undo_attention() -> None:
    try:
        from vllm.v1.attention.backends import registry

        registry._ATTN_OVERRIDES.pop(registry.AttentionBackendEnum.CUSTOM, None)
    except Exception as e:  # pragma: no cover
        logger.warning("Attention rollback failed: %s", e)


def _undo_sampler() -> None:
    try:
        from vllm.v1.sample.sampler import Sampler

        if getattr(Sampler, "_fxp_logprobs_patched", False):
            orig = getattr(Sampler, "_fxp_original_compute_logprobs", None)
            if orig is not None:
                Sampler.compute_logprobs = orig
            else:
                del Sampler.compute_logprobs
            Sampler._fxp_logprobs_patched = False
    except Exception as e:  # pragma: no cover
        logger.warning("Sampler rollback failed: %s", e)
