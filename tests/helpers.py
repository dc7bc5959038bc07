"""Shared test helpers: device primitives for the oracle, seeded inputs."""

from __future__ import annotations

import torch

from oracle import fxp_oracle as O


def device_prims(device="cuda") -> O.Prims:
    """Oracle primitives evaluated by the CUDA library's own device functions
    (``fxpr_probe_prims``), so oracle and kernels agree bit for bit on the
    float steps the reference leaves to the GPU compiler."""
    from fxpr_vllm import _native as N

    def run(op, a, b=None):
        a32 = a.to(torch.float32).contiguous()
        shape = a32.shape
        if b is not None:
            a32, b32 = torch.broadcast_tensors(a32, b.to(torch.float32))
            shape = a32.shape
            a32, b32 = a32.contiguous(), b32.contiguous()
        da = a32.to(device)
        db = b32.to(device) if b is not None else None
        out = torch.empty_like(da)
        rc = N.load().fxpr_probe_prims(op, da.data_ptr(), N.ptr(db), out.data_ptr(), da.numel(),
                                       N.stream_ptr(da.device))
        N.check(rc, "probe")
        return out.cpu().view(shape)

    return O.Prims(
        exp2=lambda x: run(0, x),
        div=lambda a, b: run(1, a, b),
        sqrt=lambda x: run(2, x),
        tanh=lambda x: run(3, x),
        exp=lambda x: run(4, x),
        log=lambda x: run(5, x),
        muladd=O.fma32,  # Triton on the GPU contracts the ALiBi multiply-add
        div_const=O.mul_rcp32,  # and divides by the constant softcap via its reciprocal
    )


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality (NaN patterns included) of two float tensors."""
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    it = {2: torch.int16, 4: torch.int32, 8: torch.int64}[a.element_size()]
    return torch.equal(a.contiguous().view(it), b.contiguous().view(it))


def paged_inputs(qlens, seqlens, H, KVH, D, page, dtype=torch.bfloat16, seed=0, extra_blocks=3):
    """Random paged-attention inputs (CPU tensors): block table is a random
    permutation of a block pool, like the decode-attention benchmark."""
    g = torch.Generator().manual_seed(seed)
    R = len(qlens)
    T = sum(qlens)
    max_blocks = max((s + page - 1) // page for s in seqlens)
    nblk = R * max_blocks + extra_blocks
    perm = torch.randperm(nblk, generator=g)
    block_table = perm[: R * max_blocks].view(R, max_blocks).to(torch.int32)
    q = torch.randn(T, H, D, generator=g).to(dtype)
    kv = torch.randn(nblk, 2, page, KVH, D, generator=g).to(dtype)
    qsl = torch.zeros(R + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(torch.tensor(qlens), 0)
    sl = torch.tensor(seqlens, dtype=torch.int32)
    return q, kv, qsl, sl, block_table
