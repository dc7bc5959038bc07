"""Paged decode attention at the full decode-attention benchmark shape:
64 requests, 32 query / 8 KV heads, head_dim 128, context U[512, 8192], page
16, block tables a random permutation of a 40k-block pool, frac_bits 16,
seed 2 -- built by the same generator as bench.py.

* every device path (chunked workspace path, cluster path) and every KV-split
  count 1/4/8/16 gives the same bits, for all 64 requests;
* a spread of requests (shortest, longest, around the 512-key work units,
  and others) is bit-exact against the oracle, whose float primitives are the
  library's device primitives (reference fixed_point_kernels/attention.py:398-489).
"""

import pytest
import torch

import bench
from oracle import fxp_oracle as O
from tests.helpers import bits_equal, device_prims

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg():
    inp = bench.attention_inputs(seed=2)
    dev = {k: v.cuda() for k, v in inp.items()}
    return inp, dev


def _run(dev, bits, splits, use_workspace=True):
    from fxpr_vllm.fixed_point_kernels import attention as A

    o = torch.zeros(dev["Q"].shape, dtype=torch.float32, device="cuda")
    A.unified_attention_fxp(dev["Q"], dev["KV"], o, dev["qsl"], dev["seq_lens"], dev["bt"], 1,
                            fxp_dtype=bits, frac_bits=16, num_kv_splits=splits,
                            max_seq_len=8192, use_workspace=use_workspace)
    return o.cpu()


def _pick_requests(seq_lens, n):
    """Shortest, longest, the ones closest to a 512-key boundary (either side),
    then evenly spaced others."""
    sl = seq_lens.tolist()
    order = sorted(range(len(sl)), key=lambda r: sl[r])
    picks = [order[0], order[-1]]
    near = sorted(range(len(sl)), key=lambda r: min(sl[r] % 512, 512 - sl[r] % 512))
    for r in near:
        if len(picks) >= 4:
            break
        if r not in picks:
            picks.append(r)
    for r in order[:: max(1, len(order) // n)]:
        if len(picks) >= n:
            break
        if r not in picks:
            picks.append(r)
    return picks


def _oracle_rows(inp, reqs, bits, prims):
    q = inp["Q"][reqs]
    sl = inp["seq_lens"][reqs]
    bt = inp["bt"][reqs]
    qsl = torch.arange(len(reqs) + 1, dtype=torch.int32)
    o = torch.zeros(q.shape, dtype=torch.float32)
    return O.unified_attention_fxp(q, inp["KV"], o, qsl, sl, bt, 1, int_bits=bits, frac_bits=16,
                                   prims=prims)


@pytest.mark.parametrize("bits,n_oracle", [(32, 12), (64, 8)])
def test_config3_paths_splits_and_oracle(cfg, bits, n_oracle):
    inp, dev = cfg
    base = _run(dev, bits, 8)
    for splits in (1, 4, 16):
        assert bits_equal(_run(dev, bits, splits), base), f"splits={splits} differs from splits=8"
    assert bits_equal(_run(dev, bits, 8, use_workspace=False), base), "cluster path differs"
    reqs = _pick_requests(inp["seq_lens"], n_oracle)
    exp = _oracle_rows(inp, reqs, bits, device_prims())
    got = base[reqs]
    for i, r in enumerate(reqs):
        assert bits_equal(got[i], exp[i]), (r, int(inp["seq_lens"][r]),
                                            (got[i] - exp[i]).abs().max().item())
