"""Plugin registration: idempotent, env-gated, transactional (reference:
register.py:15-117), plus the fixed_point_det config API."""

import pytest


@pytest.fixture
def fresh_register(monkeypatch):
    from fxpr_vllm import register as R
    from fxpr_vllm.vllm_modules import config as C

    monkeypatch.setattr(R, "_registered", False)
    old = C._runtime_config
    yield R
    C._runtime_config = old
    R._undo_sampler()
    R._undo_attention()
    R._registered = False


def test_register_idempotent_and_binds_components(fresh_register):
    R = fresh_register
    R.register()
    R.register()
    import vllm.model_executor.layers.layernorm as L
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    from vllm.v1.sample.sampler import Sampler

    assert L.RMSNorm.__name__ == "DeterministicRMSNorm"
    assert AttentionBackendEnum.CUSTOM.get_class().get_name() == "CUSTOM"
    assert getattr(Sampler, "_fxp_logprobs_patched", False)


def test_register_rolls_back_on_failure(fresh_register, monkeypatch):
    R = fresh_register
    from fxpr_vllm import monkey_patches as M
    from vllm.v1.sample.sampler import Sampler

    def boom():
        raise RuntimeError("injected failure")

    monkeypatch.setattr(M, "patch_sampler", boom)
    with pytest.raises(RuntimeError, match="injected"):
        R.register()
    assert R._registered is False
    from vllm.v1.attention.backends import registry

    assert registry.AttentionBackendEnum.CUSTOM not in registry._ATTN_OVERRIDES
    assert not getattr(Sampler, "_fxp_logprobs_patched", False)


def test_register_respects_disable_knobs(fresh_register, monkeypatch):
    R = fresh_register
    from fxpr_vllm.vllm_modules import config as C
    from vllm.v1.sample.sampler import Sampler

    monkeypatch.setenv("VLLM_FXP_DET_LOGPROBS", "0")
    C._runtime_config = None
    R.register()
    assert not getattr(Sampler, "_fxp_logprobs_patched", False)


def test_fixed_point_config_api():
    from fxpr_vllm.vllm_modules.quantisation_config import FixedPointConfig, FixedPointLinearMethod
    from vllm.model_executor.layers.linear import ReplicatedLinear
    from vllm.model_executor.layers.quantization import get_quantization_config

    assert get_quantization_config("fixed_point_det") is FixedPointConfig
    cfg = FixedPointConfig.from_config({"frac_bits": 12})
    assert cfg.frac_bits == 12 and cfg.get_name() == "fixed_point_det"
    with pytest.raises(ValueError):
        FixedPointConfig(frac_bits=40)
    import torch.nn as nn

    assert cfg.get_quant_method(nn.Linear(2, 2), "x") is None
    assert isinstance(FixedPointLinearMethod(cfg), FixedPointLinearMethod)


def test_lm_head_routed_to_fixed_point(monkeypatch):
    """The LM head gets the fixed-point logits method (an addition to the
    reference, gated by VLLM_FXP_DET_LM_HEAD); embeddings keep vLLM's own."""
    from fxpr_vllm.vllm_modules import config as C
    from fxpr_vllm.vllm_modules.quantisation_config import FixedPointConfig, FixedPointLMHeadMethod
    from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead, VocabParallelEmbedding

    head = ParallelLMHead.__new__(ParallelLMHead)
    emb = VocabParallelEmbedding.__new__(VocabParallelEmbedding)
    old = C._runtime_config
    try:
        C._runtime_config = C.FxpRuntimeConfig()
        cfg = FixedPointConfig(16)
        assert isinstance(cfg.get_quant_method(head, "lm_head"), FixedPointLMHeadMethod)
        assert cfg.get_quant_method(emb, "embed_tokens") is None
        C._runtime_config = C.FxpRuntimeConfig(enable_lm_head=False)
        assert cfg.get_quant_method(head, "lm_head") is None
    finally:
        C._runtime_config = old
