"""Row-parallel fixed-point partials reduced as integers are bitwise equal to
the TP=1 result for any TP degree (host logic on CPU ranks with gloo)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fxp_oracle as O


def _worker(rank, world, port, bits, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fxpr_vllm.vllm_modules.tp_allreduce import integer_all_reduce

        g = torch.Generator().manual_seed(0)
        x = (torch.randn(6, 96, generator=g) * 2).to(torch.bfloat16)
        w = (torch.randn(40, 96, generator=g) * 0.05).to(torch.bfloat16)
        bias = torch.randn(40, generator=g).to(torch.bfloat16)
        ks = 96 // world
        xs, ws = x[:, rank * ks:(rank + 1) * ks], w[:, rank * ks:(rank + 1) * ks]
        part = O.gemm_fxp_int(xs, ws.t(), 16, bits)  # this rank's integer partial
        part = part.to(torch.int64 if bits == 64 else torch.int32)
        total = integer_all_reduce(part, group=dist.group.WORLD)
        out = (O.fixed_to_float(O.wrap_int(total, bits), 16) + bias.float()).to(torch.bfloat16)
        ref = O.linear_apply(x, w, bias, 16, bits)  # TP=1
        q.put((rank, torch.equal(out, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("bits", [16, 32, 64])
def test_integer_allreduce_tp_invariant(world, bits):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + world * 10 + bits
    procs = [ctx.Process(target=_worker, args=(r, world, port, bits, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
