"""VLLM_FXP_* knobs: defaults, validation with warn-and-fallback
(reference: vllm_modules/config.py:51-95)."""

import pytest

from fxpr_vllm.vllm_modules import config as C


@pytest.fixture(autouse=True)
def _clean_env(monkeypatch):
    for k in ("VLLM_FXP_FRAC_BITS", "VLLM_FXP_INT_BITS", "VLLM_FXP_NUM_KV_SPLITS",
              "VLLM_FXP_DET_RMSNORM", "VLLM_FXP_DET_GEMM", "VLLM_FXP_DET_ATTN",
              "VLLM_FXP_DET_LOGPROBS"):
        monkeypatch.delenv(k, raising=False)


def test_defaults():
    cfg = C.load_runtime_config()
    assert (cfg.frac_bits, cfg.fxp_int_bits, cfg.num_kv_splits) == (16, 32, 8)
    assert cfg.enable_rmsnorm and cfg.enable_gemm and cfg.enable_attn and cfg.enable_logprobs


def test_valid_overrides(monkeypatch):
    monkeypatch.setenv("VLLM_FXP_INT_BITS", "64")
    monkeypatch.setenv("VLLM_FXP_FRAC_BITS", "40")
    monkeypatch.setenv("VLLM_FXP_NUM_KV_SPLITS", "4")
    monkeypatch.setenv("VLLM_FXP_DET_ATTN", "off")
    cfg = C.load_runtime_config()
    assert (cfg.fxp_int_bits, cfg.frac_bits, cfg.num_kv_splits) == (64, 40, 4)
    assert not cfg.enable_attn


@pytest.mark.parametrize("name,val,field,default", [
    ("VLLM_FXP_INT_BITS", "24", "fxp_int_bits", 32),
    ("VLLM_FXP_INT_BITS", "abc", "fxp_int_bits", 32),
    ("VLLM_FXP_FRAC_BITS", "32", "frac_bits", 16),
    ("VLLM_FXP_FRAC_BITS", "-1", "frac_bits", 16),
    ("VLLM_FXP_NUM_KV_SPLITS", "0", "num_kv_splits", 8),
])
def test_invalid_values_fall_back(monkeypatch, caplog, name, val, field, default):
    monkeypatch.setenv(name, val)
    cfg = C.load_runtime_config()
    assert getattr(cfg, field) == default
    assert any("fxpr_vllm" == r.name for r in caplog.records) or caplog.text


def test_singleton_and_override():
    cfg = C.FxpRuntimeConfig(frac_bits=12)
    old = C.get_runtime_config()
    try:
        C.set_runtime_config(cfg)
        assert C.get_runtime_config() is cfg
    finally:
        C.set_runtime_config(old)
