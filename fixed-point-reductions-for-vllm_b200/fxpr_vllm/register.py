"""Plugin entry point (reference: fxpr_vllm/register.py:15-117).

``register()`` is vLLM's general-plugin hook (``vllm.general_plugins``:
``fxpr_vllm = fxpr_vllm.register:register``). Its contract, kept from the
reference: it is idempotent, each component is gated by its
``VLLM_FXP_DET_*`` switch, and it is all-or-nothing -- if installing one
component fails, the components installed before it are removed again and
the error propagates. Importing this module registers the
``fixed_point_det`` quantisation method.

Here the components are rows of a table (``COMPONENTS``: switch, label,
install, uninstall) applied inside an ``_Installation``, which remembers
what it installed and unwinds it in reverse order on failure.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Callable

from . import monkey_patches
from .vllm_modules import quantisation_config  # noqa: F401  (registers fixed_point_det)
from .vllm_modules.config import FxpRuntimeConfig, get_runtime_config

logger = logging.getLogger("fxpr_vllm")

_registered = False


# ------------------------------------------------------------------ uninstallers
def _undo_rms_norm() -> None:
    try:
        import vllm.model_executor.layers.layernorm as layernorm_mod
        from vllm.model_executor.custom_op import op_registry

        op_registry.pop("rms_norm", None)
        if hasattr(layernorm_mod.RMSNorm, "_fxp_frac_bits"):  # our subclass: restore its base
            layernorm_mod.RMSNorm = layernorm_mod.RMSNorm.__mro__[1]
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

        if not getattr(Sampler, "_fxp_logprobs_patched", False):
            return
        original = getattr(Sampler, "_fxp_original_compute_logprobs", None)
        if original is None:
            del Sampler.compute_logprobs
        else:
            Sampler.compute_logprobs = original
        Sampler._fxp_logprobs_patched = False
    except Exception as e:  # pragma: no cover
        logger.warning("Sampler rollback failed: %s", e)


def _nothing() -> None:
    """The linear method is registered when quantisation_config is imported,
    so the GEMM component has nothing to install or remove."""


# ------------------------------------------------------------------ components
@dataclass(frozen=True)
class Component:
    switch: str  # FxpRuntimeConfig field that enables it
    label: str   # name used in the log lines
    install: Callable[[], object]
    uninstall: Callable[[], None]


COMPONENTS = (
    Component("enable_rmsnorm", "RMSNorm", lambda: monkey_patches.patch_rms_norm(), _undo_rms_norm),
    Component("enable_gemm", "GEMM (fixed_point_det)", _nothing, _nothing),
    Component("enable_attn", "Attention", lambda: monkey_patches.patch_attention_backend(),
              _undo_attention),
    Component("enable_logprobs", "Sampler", lambda: monkey_patches.patch_sampler(), _undo_sampler),
)


class _Installation:
    """Installs components one by one; on an exception inside the ``with``
    block, uninstalls the installed ones newest first, then lets it propagate."""

    def __init__(self) -> None:
        self._installed: list[Component] = []
        self.current: Component | None = None

    def add(self, comp: Component) -> None:
        self.current = comp
        comp.install()
        self._installed.append(comp)
        logger.info("%s registered", comp.label)

    def __enter__(self) -> "_Installation":
        return self

    def __exit__(self, exc_type, exc, tb) -> bool:
        if exc is None:
            return False
        label = self.current.label if self.current is not None else "?"
        logger.error("Error during %s registration: %s; rolling back", label, exc)
        while self._installed:
            comp = self._installed.pop()
            try:
                comp.uninstall()
            except Exception as undo_err:
                logger.error("Rollback step failed: %s", undo_err)
        return False


def _log_config(cfg: FxpRuntimeConfig) -> None:
    logger.info("Runtime Config: frac_bits=%d fxp_int_bits=%d num_kv_splits=%d rmsnorm=%s "
                "gemm=%s attn=%s logprobs=%s", cfg.frac_bits, cfg.fxp_int_bits,
                cfg.num_kv_splits, cfg.enable_rmsnorm, cfg.enable_gemm, cfg.enable_attn,
                cfg.enable_logprobs)


def register() -> None:
    """Install the deterministic components into vLLM (safe to call repeatedly)."""
    global _registered
    if _registered:
        return
    _registered = True
    try:
        cfg = get_runtime_config()
        _log_config(cfg)
        from . import _native, library_ops  # noqa: F401

        _native.load()  # fail loudly now if the CUDA library is missing
        with _Installation() as inst:
            for comp in COMPONENTS:
                if getattr(cfg, comp.switch):
                    inst.add(comp)
                else:
                    logger.info("%s registration skipped (disabled)", comp.label)
    except BaseException:
        _registered = False
        raise
