"""Pins the library's fp32 device primitives against Triton 3.6 on the same
GPU: the reference kernels use ``tl.math.exp2`` (attention.py:237), ``/``
(attention.py:268, rms_norm.py:56-57), ``tl.sqrt`` (rms_norm.py:57),
``libdevice.tanh`` (attention.py:130), ``tl.exp`` and ``tl.log``
(softmax.py:38, 44), whose rounding is whatever Triton lowers them to.
Triton is used here only as the oracle of those primitives."""

import pytest
import torch

pytestmark = pytest.mark.gpu

triton = pytest.importorskip("triton")
tl = triton.language


@triton.jit
def _prim_kernel(a_ptr, b_ptr, o_ptr, n, OP: tl.constexpr, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = offs < n
    a = tl.load(a_ptr + offs, mask=m, other=1.0)
    b = tl.load(b_ptr + offs, mask=m, other=1.0)
    if OP == 0:
        r = tl.math.exp2(a)
    elif OP == 1:
        r = a / b
    elif OP == 2:
        r = tl.sqrt(a)
    elif OP == 3:
        r = tl.extra.cuda.libdevice.tanh(a)
    elif OP == 4:
        r = tl.exp(a)
    else:
        r = tl.log(a)
    tl.store(o_ptr + offs, r, mask=m)


def _inputs(op, n=1 << 22):
    g = torch.Generator(device="cuda").manual_seed(op)
    if op == 0:
        return torch.rand(n, device="cuda", generator=g) * -40.0, None
    if op == 1:
        a = torch.randn(n, device="cuda", generator=g) * torch.exp2(torch.randint(-20, 20, (n,), device="cuda", generator=g).float())
        b = torch.rand(n, device="cuda", generator=g) * 1e4 + 1e-6
        return a, b
    if op in (2, 5):
        return torch.rand(n, device="cuda", generator=g) * torch.exp2(torch.randint(-30, 30, (n,), device="cuda", generator=g).float()), None
    if op == 3:
        return torch.randn(n, device="cuda", generator=g) * 3, None
    return torch.rand(n, device="cuda", generator=g) * -30.0, None


@pytest.mark.parametrize("op,name", [(0, "exp2"), (1, "div"), (2, "sqrt"), (3, "tanh"), (4, "exp"), (5, "log")])
def test_device_primitive_matches_triton(op, name):
    from fxpr_vllm import _native as N

    a, b = _inputs(op)
    bb = b if b is not None else torch.ones_like(a)
    ref = torch.empty_like(a)
    _prim_kernel[(triton.cdiv(a.numel(), 1024),)](a, bb, ref, a.numel(), OP=op, BLOCK=1024)
    out = torch.empty_like(a)
    rc = N.load().fxpr_probe_prims(op, a.data_ptr(), bb.data_ptr(), out.data_ptr(), a.numel(),
                                   N.stream_ptr(a.device))
    N.check(rc, "probe")
    torch.cuda.synchronize()
    mism = (ref.view(torch.int32) != out.view(torch.int32)).sum().item()
    assert mism == 0, f"{name}: {mism} of {a.numel()} differ from Triton"
