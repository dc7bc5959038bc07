"""torch.library op boundary (reference: fxpr_vllm/library_ops.py:14-126).

The three reference schemas are registered unchanged in namespace ``fxpr``:

* ``fxpr::gemm_fxp(Tensor a, Tensor b, int frac_bits, int fxp_int_bits) -> Tensor``
* ``fxpr::rms_norm_fxp(Tensor x, Tensor weight_fp32, float eps, int frac_bits, int fxp_int_bits) -> Tensor``
* ``fxpr::rms_norm_fxp_residual(Tensor x, Tensor(a!) residual, Tensor weight_fp32, float eps, int frac_bits, int fxp_int_bits) -> Tensor``

plus the ops this build adds (integer GEMM partials for the tensor-parallel
integer allreduce, its epilogue, the casts, the row sum, attention and
log-softmax). Each has a CUDA implementation only (calls into the C ABI on
the current stream, no host sync) and a fake implementation for tracing;
there is no CPU implementation, so CPU tensors fail loudly.
"""

from __future__ import annotations

import torch

from .fixed_point_kernels import attention as _attn
from .fixed_point_kernels import fixed_point as _fp
from .fixed_point_kernels import gemm as _gemm
from .fixed_point_kernels import rms_norm as _rms
from .fixed_point_kernels import softmax as _sm


@torch.library.custom_op("fxpr::gemm_fxp", mutates_args=(), device_types="cuda")
def gemm_fxp(a: torch.Tensor, b: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    return _gemm.gemm_fxp(a, b, frac_bits, fxp_int_bits)


@gemm_fxp.register_fake
def _(a, b, frac_bits, fxp_int_bits):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=torch.float32)


@torch.library.custom_op("fxpr::gemm_fxp_int", mutates_args=(), device_types="cuda")
def gemm_fxp_int(a: torch.Tensor, b: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    return _gemm.gemm_fxp_int(a, b, frac_bits, fxp_int_bits)


@gemm_fxp_int.register_fake
def _(a, b, frac_bits, fxp_int_bits):
    dt = torch.int64 if fxp_int_bits == 64 else torch.int32
    return a.new_empty((a.shape[0], b.shape[1]), dtype=dt)


@torch.library.custom_op("fxpr::fixed_to_float_bias", mutates_args=(), device_types="cuda")
def fixed_to_float_bias(acc: torch.Tensor, bias: torch.Tensor | None, frac_bits: int,
                        fxp_int_bits: int, out_dtype: torch.dtype) -> torch.Tensor:
    return _gemm.fixed_to_float_bias(acc, frac_bits, fxp_int_bits, bias, out_dtype)


@fixed_to_float_bias.register_fake
def _(acc, bias, frac_bits, fxp_int_bits, out_dtype):
    return acc.new_empty(acc.shape, dtype=out_dtype)


@torch.library.custom_op("fxpr::rms_norm_fxp", mutates_args=(), device_types="cuda")
def rms_norm_fxp(x: torch.Tensor, weight_fp32: torch.Tensor, eps: float, frac_bits: int,
                 fxp_int_bits: int) -> torch.Tensor:
    return _rms.rms_norm_fxp(x, weight_fp32, eps, frac_bits, fxp_int_bits)


@rms_norm_fxp.register_fake
def _(x, weight_fp32, eps, frac_bits, fxp_int_bits):
    return torch.empty_like(x)


@torch.library.custom_op("fxpr::rms_norm_fxp_residual", mutates_args=("residual",), device_types="cuda")
def rms_norm_fxp_residual(x: torch.Tensor, residual: torch.Tensor, weight_fp32: torch.Tensor,
                          eps: float, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    """Fused residual + RMSNorm; residual is overwritten with x + residual."""
    assert x.shape == residual.shape, "x and residual must share shape"
    return _rms.rms_norm_fxp(x, weight_fp32, eps, frac_bits, fxp_int_bits, residual=residual)


@rms_norm_fxp_residual.register_fake
def _(x, residual, weight_fp32, eps, frac_bits, fxp_int_bits):
    return torch.empty_like(x)


@torch.library.custom_op("fxpr::float_to_fixed", mutates_args=(), device_types="cuda")
def float_to_fixed(x: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    return _fp.float_to_fixed(x, frac_bits, fxp_int_bits)


@float_to_fixed.register_fake
def _(x, frac_bits, fxp_int_bits):
    return x.new_empty(x.shape, dtype=_fp.fixed_tl_dtype(fxp_int_bits))


@torch.library.custom_op("fxpr::fixed_to_float", mutates_args=(), device_types="cuda")
def fixed_to_float(q: torch.Tensor, frac_bits: int, out_dtype: torch.dtype) -> torch.Tensor:
    return _fp.fixed_to_float(q, frac_bits, out_dtype)


@fixed_to_float.register_fake
def _(q, frac_bits, out_dtype):
    return q.new_empty(q.shape, dtype=out_dtype)


@torch.library.custom_op("fxpr::fxp_sum", mutates_args=(), device_types="cuda")
def fxp_sum(x: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    return _fp.fxp_sum(x, frac_bits, fxp_int_bits)


@fxp_sum.register_fake
def _(x, frac_bits, fxp_int_bits):
    return x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("fxpr::unified_attention_fxp", mutates_args=("o",), device_types="cuda")
def unified_attention_fxp(q: torch.Tensor, kv_cache: torch.Tensor, o: torch.Tensor,
                          query_start_loc: torch.Tensor, seq_lens: torch.Tensor,
                          block_table: torch.Tensor, max_query_len: int,
                          alibi_slopes: torch.Tensor | None, fxp_int_bits: int, is_causal: bool,
                          softmax_scale: float | None, frac_bits: int, logits_soft_cap: float,
                          window_size: int, num_kv_splits: int, max_seq_len: int) -> None:
    _attn.unified_attention_fxp(q, kv_cache, o, query_start_loc, seq_lens, block_table,
                                max_query_len, alibi_slopes=alibi_slopes, fxp_dtype=fxp_int_bits,
                                is_causal=is_causal, softmax_scale=softmax_scale,
                                frac_bits=frac_bits, logits_soft_cap=logits_soft_cap,
                                window_size=window_size, num_kv_splits=num_kv_splits,
                                max_seq_len=max_seq_len or None)


@unified_attention_fxp.register_fake
def _(q, kv_cache, o, query_start_loc, seq_lens, block_table, max_query_len, alibi_slopes,
      fxp_int_bits, is_causal, softmax_scale, frac_bits, logits_soft_cap, window_size,
      num_kv_splits, max_seq_len):
    return None


@torch.library.custom_op("fxpr::log_softmax_fxp", mutates_args=(), device_types="cuda")
def log_softmax_fxp(x: torch.Tensor, fxp_int_bits: int, dim: int, frac_bits: int) -> torch.Tensor:
    return _sm.log_softmax_fxp(x, fxp_int_bits, dim=dim, frac_bits=frac_bits)


@log_softmax_fxp.register_fake
def _(x, fxp_int_bits, dim, frac_bits):
    return torch.empty_like(x)


@torch.library.custom_op("fxpr::fixed_to_float_add_rms_norm", mutates_args=("residual",),
                         device_types="cuda")
def fixed_to_float_add_rms_norm(acc: torch.Tensor, bias: torch.Tensor | None, residual: torch.Tensor,
                                weight: torch.Tensor, eps: float, frac_bits: int,
                                fxp_int_bits: int) -> torch.Tensor:
    return _rms.fixed_to_float_add_rms_norm(acc, bias, residual, weight, eps, frac_bits, fxp_int_bits)


@fixed_to_float_add_rms_norm.register_fake
def _(acc, bias, residual, weight, eps, frac_bits, fxp_int_bits):
    return torch.empty_like(residual)
