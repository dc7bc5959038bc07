"""The CPU oracle against golden vectors produced by the reference's own
Triton kernels (tests/golden/make_golden.py), and against the known-answer
tests of the reference's test suite (tests/test_fixed_point_cast.py,
tests/test_sum.py in the reference project)."""

import os

import pytest
import torch

from oracle import fxp_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLD, name), weights_only=False)


def test_casts_match_reference_kernels():
    n = 0
    for c in _load("casts.pt"):
        if c["kind"] == "f2x":
            got = O.float_to_fixed(c["x"], c["frac"], c["bits"])
            exp = c["out"]
            if c["x"].dtype == torch.float64:
                # the Triton interpreter casts out-of-range values with numpy
                # (wraps); the GPU conversion saturates. Pin those separately.
                over = (c["x"].abs() * 2.0 ** c["frac"]) >= 2.0 ** (c["bits"] - 1)
                info = torch.iinfo(got.dtype)
                sat = torch.where(c["x"] > 0, torch.tensor(info.max), torch.tensor(info.min)).to(got.dtype)
                assert torch.equal(got[over], sat[over])
                got, exp = got[~over], exp[~over]
            assert torch.equal(got, exp), (c["bits"], c["frac"])
        else:
            fdt = getattr(torch, c["fdt"].split(".")[1])
            assert torch.equal(O.fixed_to_float(c["x"], c["frac"], fdt), c["out"])
        n += 1
    assert n == 36


def test_gemm_matches_reference_kernel():
    for c in _load("gemm.pt"):
        assert torch.equal(O.gemm_fxp(c["a"], c["b"], c["frac"], c["bits"]), c["out"])


def test_rms_norm_matches_reference_kernel():
    for c in _load("rms_norm.pt"):
        r = O.rms_norm_fxp(c["x"], c["w"], c["eps"], c["frac"], c["bits"], residual=c["residual"])
        if c["residual"] is not None:
            y, res = r
            assert torch.equal(res, c["residual_out"])
        else:
            y = r
        assert torch.equal(y, c["out"])


def test_attention_matches_reference_kernel():
    for c in _load("attention.pt"):
        o = torch.zeros_like(c["out"])
        slopes = c["alibi_slopes"] * O.RCP_LN2 if c["alibi_slopes"] is not None else None
        O.unified_attention_fxp(c["q"], c["kv_cache"], o, c["query_start_loc"], c["seq_lens"],
                                c["block_table"], c["max_query_len"], alibi_slopes=slopes,
                                int_bits=c["bits"], is_causal=c["causal"], frac_bits=c["frac"],
                                logits_soft_cap=c["softcap"], window_size=c["window"])
        assert torch.equal(o, c["out"])


def test_log_softmax_matches_reference_kernel():
    for c in _load("log_softmax.pt"):
        assert torch.equal(O.log_softmax_fxp(c["x"], c["bits"], c["frac"]), c["out"])


# ---- known answers from the reference's test suite ----

def test_cast_known_values_q16_16():
    x = torch.tensor([0.0, 1.0, -1.0, 0.5, -0.5, 0.25, 1.5, -1.5, 2**15 - 1, -(2**15)])
    exp = torch.tensor([0, 1 << 16, -(1 << 16), 1 << 15, -(1 << 15), 1 << 14, (1 << 16) + (1 << 15),
                        -((1 << 16) + (1 << 15)), (2**15 - 1) << 16, -(2**15) << 16], dtype=torch.int32)
    assert torch.equal(O.float_to_fixed(x, 16, 32), exp)


def test_cast_saturation():
    got = O.float_to_fixed(torch.tensor([1e30, -1e30, 0.0]), 0, 32)
    imax, imin = torch.iinfo(torch.int32).max, torch.iinfo(torch.int32).min
    assert imax - 256 <= got[0].item() <= imax
    assert imin <= got[1].item() <= imin + 256
    assert got[2].item() == 0


def test_cast_nan_maps_to_qmin():
    assert O.float_to_fixed(torch.tensor([float("nan")]), 16, 32).item() == -(2**31)


@pytest.mark.parametrize("frac_bits", [0, 4, 16])
def test_roundtrip_lossless(frac_bits):
    c = torch.tensor([0.0, 1.0, -1.0, 0.5, -0.5, 0.25, 0.125, 2.0, -2.0, 10.0, -10.0])
    base = c[(c / 2**-frac_bits).frac() == 0]
    assert torch.equal(O.fixed_to_float(O.float_to_fixed(base, frac_bits, 32), frac_bits), base)


def test_sum_saturates_and_is_order_free():
    x = torch.tensor([float(1 << 30), float(1 << 30), 16.0])
    imax = O.fixed_to_float(torch.tensor(torch.iinfo(torch.int32).max), 0)
    imin = O.fixed_to_float(torch.tensor(torch.iinfo(torch.int32).min), 0)
    assert torch.equal(O.fxp_sum(x, 0, 32), imax)
    assert torch.equal(O.fxp_sum(-x, 0, 32), imin)
    a = torch.tensor([65504.0, -65504.0, 1.0])
    assert O.fxp_sum(a, 0).item() == O.fxp_sum(a[[0, 2, 1]], 0).item() == 1.0


def test_attention_int16_rejected():
    q = torch.zeros(1, 1, 32)
    kv = torch.zeros(1, 2, 16, 1, 32)
    with pytest.raises(ValueError):
        O.unified_attention_fxp(q, kv, torch.zeros_like(q), torch.tensor([0, 1]), torch.tensor([1]),
                                torch.zeros(1, 1, dtype=torch.int32), 1, int_bits=16)
