"""Q-format helpers and the elementwise cast / sum launchers.

Mirrors ``fxpr_vllm/fixed_point_kernels/fixed_point.py`` of the reference
(``RCP_LN2`` line 4, ``fixed_tl_dtype`` 9-14, ``int_bits_of`` 17-22,
``float_to_fixed`` 25-53, ``fixed_to_float`` 56-69). The reference's casts are
Triton device functions; here the same casts are CUDA device functions used
by every kernel, and these host launchers expose them elementwise.
"""

from __future__ import annotations

import torch

from .. import _native as N

RCP_LN2 = 1.4426950408889634

_INT_BY_BITS = {16: torch.int16, 32: torch.int32, 64: torch.int64}


def fixed_tl_dtype(int_bits: int) -> torch.dtype:
    """Signed integer dtype for a bit width (16/32/64); ValueError otherwise
    (fixed_point.py:9-14). Returns a torch dtype instead of a Triton dtype."""
    try:
        return _INT_BY_BITS[int_bits]
    except KeyError:
        raise ValueError(f"fxp_int_bits must be 16/32/64, got {int_bits}") from None


fixed_int_dtype = fixed_tl_dtype


def int_bits_of(fxp_dtype) -> int:
    """Inverse of :func:`fixed_tl_dtype` (fixed_point.py:17-22). Accepts a
    torch integer dtype, an int bit width, or any object with a
    ``primitive_bitwidth`` attribute (a Triton dtype)."""
    if isinstance(fxp_dtype, int):
        bits = fxp_dtype
    elif isinstance(fxp_dtype, torch.dtype):
        bits = {torch.int16: 16, torch.int32: 32, torch.int64: 64}.get(fxp_dtype)
    else:
        bits = getattr(fxp_dtype, "primitive_bitwidth", None)
    if bits not in (16, 32, 64):
        raise ValueError(f"Unsupported fxp dtype {fxp_dtype!r}")
    return bits


def float_to_fixed(x: torch.Tensor, frac_bits: int, out: torch.dtype | int = torch.int32) -> torch.Tensor:
    """Elementwise F2X: round-to-nearest-even of x*2^f with saturation, into
    ``out`` (int16/int32/int64). x must be float16/float32/float64."""
    bits = int_bits_of(out)
    dev = N.require_cuda(x)
    xc = x.contiguous()
    q = torch.empty(x.shape, dtype=_INT_BY_BITS[bits], device=dev)
    if x.dtype == torch.bfloat16:
        raise TypeError("x must be of a floating-point type float16/float32/float64")
    rc = N.load().fxpr_float_to_fixed(xc.data_ptr(), N.dcode(xc), q.data_ptr(), bits, xc.numel(),
                                      frac_bits, N.stream_ptr(dev))
    N.check(rc, "float_to_fixed")
    return q


def fixed_to_float(q: torch.Tensor, frac_bits: int, out: torch.dtype = torch.float32) -> torch.Tensor:
    """Elementwise X2F: ``q.to(out) * 2^-f`` (RNE conversion)."""
    bits = int_bits_of(q.dtype)
    dev = N.require_cuda(q)
    qc = q.contiguous()
    y = torch.empty(q.shape, dtype=out, device=dev)
    rc = N.load().fxpr_fixed_to_float(qc.data_ptr(), bits, y.data_ptr(), N.dcode(y), qc.numel(),
                                      frac_bits, N.stream_ptr(dev))
    N.check(rc, "fixed_to_float")
    return y


def fxp_sum(x: torch.Tensor, frac_bits: int, fxp_int_bits: int = 32) -> torch.Tensor:
    """Fixed-point sum over the last dim (fp32 result): per-element F2X into
    int_b, exact integer sum, saturation to the int_b range, X2F. Same
    semantics as the reference's ``fixed_sum_as_float`` (tests/test_sum.py:13-29)."""
    bits = int_bits_of(fxp_int_bits)
    dev = N.require_cuda(x)
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() > 0 else x.reshape(1, 1)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty(x2.shape[0], dtype=torch.float32, device=dev)
    rc = N.load().fxpr_fxp_sum(x2.data_ptr(), N.dcode(x2), x2.shape[0], x2.shape[1], x2.stride(0),
                               out.data_ptr(), frac_bits, bits, N.stream_ptr(dev))
    N.check(rc, "fxp_sum")
    return out.view(x.shape[:-1])
