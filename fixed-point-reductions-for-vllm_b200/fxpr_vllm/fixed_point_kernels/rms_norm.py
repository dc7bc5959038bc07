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
