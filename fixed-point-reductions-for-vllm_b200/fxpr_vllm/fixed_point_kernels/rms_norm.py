"""Fixed-point RMSNorm launcher (reference: fixed_point_kernels/rms_norm.py:10-60,
library_ops.py:53-126)."""

from __future__ import annotations

import torch

from .. import _native as N
from .fixed_point import int_bits_of


def rms_norm_fxp(x: torch.Tensor, weight: torch.Tensor, eps: float, frac_bits: int,
                 fxp_int_bits: int, residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """y = (x [+ residual]) * w * rrms with an integer squared-sum; y has x's
    dtype. With ``residual``, x + residual (fp32) is written into residual in
    place, in residual's dtype."""
    bits = int_bits_of(fxp_int_bits)
    dev = N.require_cuda(x, weight, residual)
    hidden = x.shape[-1]
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty(x2.shape, dtype=x.dtype, device=dev)
    y2 = y.view(-1, hidden)
    w = weight.contiguous()
    r2 = None
    if residual is not None:
        if residual.shape != x.shape:
            raise AssertionError("x and residual must share shape")
        r2 = residual.view(-1, hidden) if residual.is_contiguous() else residual.contiguous().view(-1, hidden)
    rc = N.load().fxpr_rms_norm_fxp(
        x2.data_ptr(), N.dcode(x2), x2.stride(0), w.data_ptr(), N.dcode(w), y2.data_ptr(),
        N.dcode(y2), y2.stride(0), N.ptr(r2), N.dcode(r2) if r2 is not None else 0,
        r2.stride(0) if r2 is not None else 0, x2.shape[0], hidden, float(eps), frac_bits, bits,
        N.stream_ptr(dev))
    N.check(rc, "rms_norm_fxp")
    if residual is not None and r2.data_ptr() != residual.data_ptr():
        residual.copy_(r2.view_as(residual))
    return y.view(x.shape)


def fixed_to_float_add_rms_norm(acc: torch.Tensor, bias: torch.Tensor | None, residual: torch.Tensor,
                                weight: torch.Tensor, eps: float, frac_bits: int,
                                fxp_int_bits: int) -> torch.Tensor:
    """One pass of: h = cast(X2F(acc) + bias) to residual's dtype (the
    row-parallel linear layer's output after the integer allreduce), residual
    += h in fp32 (in place), y = fixed-point RMSNorm of the fp32 sum. Same bits
    as ``fixed_to_float_bias`` followed by ``rms_norm_fxp(..., residual=...)``."""
    bits = int_bits_of(fxp_int_bits)
    dev = N.require_cuda(acc, residual, weight, bias)
    hidden = acc.shape[-1]
    a2 = acc.reshape(-1, hidden)
    if a2.stride(-1) != 1:
        a2 = a2.contiguous()
    if residual.shape != acc.shape or not residual.is_contiguous():
        raise AssertionError("residual must be a contiguous tensor of acc's shape")
    r2 = residual.view(-1, hidden)
    y = torch.empty(r2.shape, dtype=residual.dtype, device=dev)
    w = weight.contiguous()
    b = bias.contiguous() if bias is not None else None
    rc = N.load().fxpr_fixed_to_float_add_rms_norm(
        a2.data_ptr(), bits, a2.stride(0), N.ptr(b), N.dcode(b) if b is not None else 0,
        r2.data_ptr(), N.dcode(r2), r2.stride(0), w.data_ptr(), N.dcode(w), y.data_ptr(), y.stride(0),
        a2.shape[0], hidden, float(eps), frac_bits, N.stream_ptr(dev))
    N.check(rc, "fixed_to_float_add_rms_norm")
    return y.view(residual.shape)
