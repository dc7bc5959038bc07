"""Fixed-point GEMM launcher (reference: fixed_point_kernels/gemm.py:97-196,
library_ops.py:14-45).

``C = X2F(sum_k F2X(fp32(a[m,k]) * fp32(b[k,n])))``; b is ``[K, N]`` with any
strides (the linear method passes the nn.Linear weight ``[N, K]`` as the
transposed view, which the kernel reads K-contiguous without a copy).
"""

from __future__ import annotations

import torch

from .. import _native as N
from .fixed_point import int_bits_of


def _gemm(a: torch.Tensor, b: torch.Tensor, frac_bits: int, fxp_int_bits: int,
          out_int: bool) -> torch.Tensor:
    bits = int_bits_of(fxp_int_bits)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise AssertionError(f"gemm_fxp: bad shapes {tuple(a.shape)} x {tuple(b.shape)}")
    dev = N.require_cuda(a, b)
    M, K = a.shape
    N_ = b.shape[1]
    if out_int:
        c = torch.empty((M, N_), dtype=torch.int64 if bits == 64 else torch.int32, device=dev)
    else:
        c = torch.empty((M, N_), dtype=torch.float32, device=dev)
    if M == 0 or N_ == 0:
        return c
    lib = N.load()
    need = lib.fxpr_gemm_workspace_bytes(M, N_, K, bits)
    ws = N.gemm_workspace(dev, need)
    rc = lib.fxpr_gemm_fxp(a.data_ptr(), N.dcode(a), a.stride(0), a.stride(1), b.data_ptr(),
                           N.dcode(b), b.stride(0), b.stride(1), c.data_ptr(), 1 if out_int else 0,
                           c.stride(0), c.stride(1), M, N_, K, frac_bits, bits,
                           N.ptr(ws), 0 if ws is None else ws.numel(), N.stream_ptr(dev))
    N.check(rc, "gemm_fxp")
    return c


def gemm_fxp(a: torch.Tensor, b: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    """fp32 ``[M, N]`` output, as ``fxpr::gemm_fxp`` (library_ops.py:14-45)."""
    return _gemm(a, b, frac_bits, fxp_int_bits, out_int=False)


def gemm_fxp_int(a: torch.Tensor, b: torch.Tensor, frac_bits: int, fxp_int_bits: int) -> torch.Tensor:
    """Raw integer accumulator (int32 for 16/32-bit, int64 for 64-bit), the
    partial a row-parallel layer allreduces before X2F."""
    return _gemm(a, b, frac_bits, fxp_int_bits, out_int=True)


def fixed_to_float_bias(acc: torch.Tensor, frac_bits: int, fxp_int_bits: int,
                        bias: torch.Tensor | None, out_dtype: torch.dtype) -> torch.Tensor:
    """``cast(X2F(acc) + fp32(bias))`` -- quantisation_config.py:181-187 after
    an integer allreduce."""
    bits = int_bits_of(fxp_int_bits)
    dev = N.require_cuda(acc, bias)
    a2 = acc.reshape(-1, acc.shape[-1])
    if a2.stride(-1) != 1:
        a2 = a2.contiguous()
    out = torch.empty(a2.shape, dtype=out_dtype, device=dev)
    b = bias.contiguous() if bias is not None else None
    rc = N.load().fxpr_fixed_to_float_bias(
        a2.data_ptr(), bits, a2.shape[0], a2.shape[1], a2.stride(0), N.ptr(b),
        N.dcode(b) if b is not None else 0, out.data_ptr(), N.dcode(out), out.stride(0),
        frac_bits, N.stream_ptr(dev))
    N.check(rc, "fixed_to_float_bias")
    return out.view(*acc.shape[:-1], acc.shape[-1])
