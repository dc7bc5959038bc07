"""Deterministic attention backend bound to vLLM's CUSTOM slot
(reference: fxpr_vllm/vllm_modules/attention_backend.py:42-228).

Metadata and its builder are vLLM's Triton-attention ones (query_start_loc,
seq_lens, block_table, max_query_len, max_seq_len); the paged KV cache layout
``[num_blocks, 2, block_size, num_kv_heads, head_size]`` and the cache update
(``reshape_and_cache_flash``) are vLLM's. The attention itself is
``unified_attention_fxp`` on the B200 kernel, split over
``VLLM_FXP_NUM_KV_SPLITS`` KV splits (results do not depend on the count).
"""

from __future__ import annotations

import logging

import torch
from vllm.v1.attention.backend import AttentionImpl, AttentionLayer, AttentionType
from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend

from ..fixed_point_kernels.attention import unified_attention_fxp
from ..fixed_point_kernels.fixed_point import RCP_LN2
from .config import get_runtime_config

logger = logging.getLogger("fxpr_vllm")


class DeterministicAttentionBackend(TritonAttentionBackend):
    """Fixed-point deterministic attention backend."""

    accept_output_buffer: bool = True
    forward_includes_kv_cache_update: bool = False

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["DeterministicAttentionImpl"]:
        return DeterministicAttentionImpl

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size in (32, 64, 128, 256)

    @classmethod
    def supports_sink(cls) -> bool:
        return False


class DeterministicAttentionImpl(AttentionImpl):
    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int,
                 alibi_slopes: list[float] | None, sliding_window: int | None,
                 kv_cache_dtype: str = "auto", logits_soft_cap: float | None = None,
                 attn_type: AttentionType | None = AttentionType.DECODER,
                 *_extra_positional, **kwargs) -> None:
        if attn_type is not None and attn_type != AttentionType.DECODER:
            raise NotImplementedError(
                f"DeterministicAttention only supports decoder attention; got attn_type={attn_type!r}.")
        if kv_cache_dtype not in ("auto", "fp16", "bf16", "float16", "bfloat16"):
            raise NotImplementedError(
                f"DeterministicAttention does not support kv_cache_dtype={kv_cache_dtype!r}; "
                "supported: auto, fp16, bf16.")
        cfg = get_runtime_config()
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.num_kv_groups = num_heads // num_kv_heads
        self.kv_cache_dtype = kv_cache_dtype
        self.logits_soft_cap = float(logits_soft_cap) if logits_soft_cap else 0.0
        self.window_size = int(sliding_window) if sliding_window else 0
        self.attn_type = attn_type or AttentionType.DECODER
        self.frac_bits = cfg.frac_bits
        self.fxp_int_bits = cfg.fxp_int_bits
        self.num_kv_splits = cfg.num_kv_splits
        if alibi_slopes is not None:
            slopes = torch.tensor(alibi_slopes, dtype=torch.float32) * RCP_LN2
            assert slopes.shape == (num_heads,), \
                f"alibi_slopes shape {tuple(slopes.shape)} != (num_heads={num_heads},)"
            self.alibi_slopes: torch.Tensor | None = slopes
        else:
            self.alibi_slopes = None

    def forward(self, layer: AttentionLayer, query: torch.Tensor, key: torch.Tensor,
                value: torch.Tensor, kv_cache: torch.Tensor, attn_metadata,
                output: torch.Tensor | None = None, output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None, **kwargs) -> torch.Tensor:
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("DeterministicAttention does not support fp8/quantized output scales.")
        num_tokens = query.shape[0]
        query = query.view(num_tokens, self.num_heads, self.head_size)
        if output is None:
            output = torch.empty(num_tokens, self.num_heads, self.head_size, dtype=query.dtype,
                                 device=query.device)
        else:
            output = output.view(num_tokens, self.num_heads, self.head_size)
        if attn_metadata is None:
            output.zero_()  # profiling run before metadata exists
            return output.view(num_tokens, self.num_heads * self.head_size)
        if self.alibi_slopes is not None and self.alibi_slopes.device != query.device:
            self.alibi_slopes = self.alibi_slopes.to(query.device)
        n = attn_metadata.num_actual_tokens
        unified_attention_fxp(
            q=query[:n], kv_cache=kv_cache, o=output[:n],
            query_start_loc=attn_metadata.query_start_loc, seq_lens=attn_metadata.seq_lens,
            block_table=attn_metadata.block_table, max_query_len=int(attn_metadata.max_query_len),
            alibi_slopes=self.alibi_slopes, fxp_dtype=self.fxp_int_bits, is_causal=True,
            softmax_scale=self.scale, frac_bits=self.frac_bits,
            logits_soft_cap=self.logits_soft_cap, window_size=self.window_size,
            num_kv_splits=self.num_kv_splits, max_seq_len=int(attn_metadata.max_seq_len),
        )
        return output.view(num_tokens, self.num_heads * self.head_size)

    def do_kv_cache_update(self, layer: AttentionLayer, key: torch.Tensor, value: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            return
        from vllm._custom_ops import reshape_and_cache_flash

        key_cache, value_cache = kv_cache.unbind(1)
        reshape_and_cache_flash(key, value, key_cache, value_cache, slot_mapping,
                                self.kv_cache_dtype, layer._k_scale, layer._v_scale)
