"""Fixed-point log-softmax launcher (reference: fixed_point_kernels/softmax.py:55-97)."""

from __future__ import annotations

import torch

from .. import _native as N
from .fixed_point import int_bits_of


def log_softmax_fxp(x: torch.Tensor, fxp_dtype=torch.int32, dim: int = -1, frac_bits: int = 16,
                    block_n: int = 1024) -> torch.Tensor:
    """Log-softmax along ``dim`` with a fixed-point exp-sum; logits are rounded
    to fp16 before the max and the exp, as in the reference."""
    bits = int_bits_of(fxp_dtype)
    dev = N.require_cuda(x)
    orig_dtype = x.dtype
    if dim < 0:
        dim += x.ndim
    transposed = dim != x.ndim - 1
    x = x.transpose(dim, -1).contiguous() if transposed else x.contiguous()
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).to(torch.float32)
    y2 = torch.empty_like(x2)
    rc = N.load().fxpr_log_softmax_fxp(x2.data_ptr(), x2.stride(0), y2.data_ptr(), y2.stride(0),
                                       x2.shape[0], x2.shape[1], frac_bits, bits, N.stream_ptr(dev))
    N.check(rc, "log_softmax_fxp")
    y = y2.view(shape).to(orig_dtype)
    if transposed:
        y = y.transpose(dim, -1).contiguous()
    return y
