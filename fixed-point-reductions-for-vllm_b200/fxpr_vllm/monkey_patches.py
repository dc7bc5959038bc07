"""vLLM hook points that have no registration API (reference: fxpr_vllm/monkey_patches.py).

* RMSNorm: model files import the ``RMSNorm`` symbol directly, so the layer
  module's symbol and every already-imported ``vllm.model_executor.models.*``
  module's symbol are rebound to :class:`DeterministicRMSNorm`.
* Attention: the backend class path is bound to ``AttentionBackendEnum.CUSTOM``.
* Sampler: ``Sampler.compute_logprobs`` is replaced by the deterministic
  log-softmax.
"""

from __future__ import annotations

import logging
import sys

logger = logging.getLogger("fxpr_vllm")


def patch_rms_norm() -> int:
    """Rebind RMSNorm everywhere it is imported; returns the number of model
    modules rebound."""
    from vllm.model_executor.custom_op import op_registry
    import vllm.model_executor.layers.layernorm as layernorm_mod

    op_registry.pop("rms_norm", None)  # the subclass registers itself under this name
    from .vllm_modules.rms_norm import DeterministicRMSNorm

    original = layernorm_mod.RMSNorm
    if original is DeterministicRMSNorm:
        return 0
    layernorm_mod.RMSNorm = DeterministicRMSNorm
    patched = 0
    for name, mod in list(sys.modules.items()):
        if mod is None or not name.startswith("vllm.model_executor.models."):
            continue
        if getattr(mod, "RMSNorm", None) is original:
            setattr(mod, "RMSNorm", DeterministicRMSNorm)
            patched += 1
    assert op_registry.get("rms_norm") in (None, DeterministicRMSNorm), (
        "rms_norm op_registry entry was clobbered by another plugin")
    if patched == 0:
        logger.warning("DeterministicRMSNorm: no vllm.model_executor.models.* module rebound "
                       "(none imported yet, or the import path changed)")
    return patched


def patch_attention_backend() -> None:
    """Bind the deterministic backend to vLLM's CUSTOM attention backend slot."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    from .vllm_modules.attention_backend import DeterministicAttentionBackend

    register_backend(AttentionBackendEnum.CUSTOM,
                     class_path=f"{DeterministicAttentionBackend.__module__}."
                                f"{DeterministicAttentionBackend.__qualname__}")


def patch_sampler() -> None:
    """Replace ``Sampler.compute_logprobs`` with the deterministic log-softmax."""
    from vllm.v1.sample.sampler import Sampler

    from .vllm_modules.sampling import deterministic_log_softmax

    if getattr(Sampler, "_fxp_logprobs_patched", False):
        return
    Sampler._fxp_original_compute_logprobs = Sampler.__dict__.get("compute_logprobs")
    Sampler.compute_logprobs = staticmethod(deterministic_log_softmax)
    Sampler._fxp_logprobs_patched = True
    logger.info("Sampler log-softmax patched")
