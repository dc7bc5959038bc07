"""Integer allreduce of row-parallel fixed-point partials.

The reference lets vLLM allreduce the *float* outputs of row-parallel layers
(``RowParallelLinear.forward``, vllm/model_executor/layers/linear.py), which
makes results depend on the TP degree. Here each rank produces its raw integer
accumulator (``fxpr::gemm_fxp_int``), the accumulators are summed as int32 /
int64 (exact and order-free, NCCL SUM over NVLink), and only then converted
with X2F + bias + cast on every rank -- bitwise identical to TP=1.
int16 accumulators travel as int32: the low 16 bits of a mod-2^32 sum are the
mod-2^16 sum.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _pynccl():
    from vllm.distributed import get_tp_group

    tp = get_tp_group()
    comm = getattr(tp, "device_communicator", None)
    pynccl = getattr(comm, "pynccl_comm", None) if comm is not None else None
    if pynccl is not None and getattr(pynccl, "disabled", True):
        pynccl = None
    return tp, pynccl


def integer_all_reduce(t: torch.Tensor, group=None) -> torch.Tensor:
    """Sum an int32/int64 tensor over a process group (exact), in place when
    possible. With ``group=None`` the vLLM tensor-parallel group is used (its
    pynccl communicator when available, which is CUDA-graph capturable)."""
    if t.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"integer_all_reduce expects int32/int64, got {t.dtype}")
    if group is not None:
        if dist.get_world_size(group) > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        return t
    tp, pynccl = _pynccl()
    if tp.world_size == 1:
        return t
    if pynccl is not None:
        out = pynccl.all_reduce(t, t)
        if out is not None:
            return out
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=tp.device_group)
    return t


@torch.library.custom_op("fxpr::integer_all_reduce", mutates_args=(), device_types="cuda")
def integer_all_reduce_op(t: torch.Tensor) -> torch.Tensor:
    """Opaque op form of :func:`integer_all_reduce` over the vLLM TP group, so
    that torch.compile and CUDA-graph capture treat it as one node (vLLM's own
    all-reduce op may route int tensors into float-only custom kernels). The
    op may not mutate its input: NCCL reduces out of place into a fresh
    buffer (no copy of the input)."""
    if t.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"integer_all_reduce expects int32/int64, got {t.dtype}")
    tp, pynccl = _pynccl()
    if tp.world_size == 1:
        return t.clone()
    if pynccl is not None:
        out = pynccl.all_reduce(t, torch.empty_like(t))
        if out is not None:
            return out
    out = t.clone()
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=tp.device_group)
    return out


@integer_all_reduce_op.register_fake
def _(t):
    return torch.empty_like(t)
