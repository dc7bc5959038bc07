"""CUDA kernels against the CPU oracle (bit-exact) on the same seeded inputs.

The oracle's float primitives are the library's own device primitives
(``helpers.device_prims``); those are pinned against Triton on the same GPU
in test_prims_triton_gpu.py.
"""

import os

import pytest
import torch

from oracle import fxp_oracle as O
from tests.helpers import bits_equal, device_prims, paged_inputs

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLD, name), weights_only=False)


@pytest.fixture(scope="module")
def prims():
    return device_prims()


# --------------------------------------------------------------------- casts
def test_casts_golden():
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    for c in _load("casts.pt"):
        if c["kind"] == "f2x":
            got = F.float_to_fixed(c["x"].cuda(), c["frac"], c["bits"]).cpu()
            assert torch.equal(got, O.float_to_fixed(c["x"], c["frac"], c["bits"]))
        else:
            fdt = getattr(torch, c["fdt"].split(".")[1])
            got = F.fixed_to_float(c["x"].cuda(), c["frac"], fdt).cpu()
            assert torch.equal(got, c["out"])


@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
def test_casts_random(bits, dtype):
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    g = torch.Generator().manual_seed(bits)
    x = torch.cat([torch.randn(5000, generator=g) * 100, torch.randn(5000, generator=g),
                   torch.tensor([0.5, 1.5, 2.5, -0.5, 1e30, -1e30, float("inf"), float("-inf"),
                                 float("nan")])]).to(dtype)
    for f in (0, 8, 14):
        got = F.float_to_fixed(x.cuda(), f, bits).cpu()
        assert torch.equal(got, O.float_to_fixed(x, f, bits)), (dtype, bits, f)


def test_cast_known_values_and_roundtrip():
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    x = torch.tensor([0.0, 1.0, -1.0, 0.5, -0.5, 0.25, 1.5, -1.5, 2**15 - 1, -(2**15)], device="cuda")
    exp = torch.tensor([0, 1 << 16, -(1 << 16), 1 << 15, -(1 << 15), 1 << 14, (1 << 16) + (1 << 15),
                        -((1 << 16) + (1 << 15)), (2**15 - 1) << 16, -(2**15) << 16],
                       dtype=torch.int32, device="cuda")
    assert torch.equal(F.float_to_fixed(x, 16, torch.int32), exp)
    q = torch.tensor([0, 1, -1, 123, -123, 1 << 20, -(1 << 20)], dtype=torch.int32, device="cuda")
    for f in (0, 8, 16):
        assert torch.equal(F.float_to_fixed(F.fixed_to_float(q, f), f, torch.int32), q)


# ----------------------------------------------------------------------- sum
@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fxp_sum(bits, dtype):
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    g = torch.Generator().manual_seed(1)
    x = (torch.randn(67, 1029, generator=g) * 3).to(dtype)
    for f in (4, 16):
        got = F.fxp_sum(x.cuda(), f, bits).cpu()
        assert torch.equal(got, O.fxp_sum(x, f, bits))


@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fxp_sum_vector_path(bits, dtype):
    """16-byte aligned rows take the vectorised magic-constant path: rows with
    a ragged tail (strided view), rows whose values force the exact path
    (large, inf, NaN) next to rows that do not."""
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    g = torch.Generator().manual_seed(11 + bits)
    base = (torch.randn(40, 1032, generator=g) * 3).to(dtype)
    base[3, 17] = 1e6
    base[5, 1000] = float("inf")
    base[7, 2] = float("-inf")
    base[9, 500] = float("nan")
    base[11, :] = 2.0 ** 14  # saturates every width's row sum
    f = 4 if bits == 16 else 16
    for view in (base, base[:, :1001], base[:, :8]):
        got = F.fxp_sum(view.cuda(), f, bits).cpu()
        assert torch.equal(got, O.fxp_sum(view, f, bits)), (view.shape, bits, dtype)


def test_fxp_sum_saturation_and_order():
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    x = torch.tensor([[float(1 << 30), float(1 << 30), 16.0]], device="cuda")
    assert torch.equal(F.fxp_sum(x, 0, 32).cpu(), O.fxp_sum(x.cpu(), 0, 32))
    a = torch.tensor([[65504.0, -65504.0, 1.0], [65504.0, 1.0, -65504.0]], device="cuda")
    s = F.fxp_sum(a, 0, 32)
    assert s[0].item() == s[1].item() == 1.0


# ---------------------------------------------------------------------- GEMM
def test_gemm_golden():
    from fxpr_vllm.fixed_point_kernels import gemm as G

    for c in _load("gemm.pt"):
        got = G.gemm_fxp(c["a"].cuda(), c["b"].cuda(), c["frac"], c["bits"]).cpu()
        assert torch.equal(got, c["out"]), (c["a"].shape, c["bits"])


def _gemm_case(M, K, N, dtype, bits, layout, sa=1.0, sb=0.02, f=16, seed=0):
    from fxpr_vllm.fixed_point_kernels import gemm as G

    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) * sa).to(dtype)
    w = (torch.randn(N, K, generator=g) * sb).to(dtype)  # nn.Linear layout
    if layout == "ncontig":
        b = w.t().contiguous()
    elif layout == "kcontig":
        b = w.t()
    else:  # strided, misaligned for cp.async
        b = torch.zeros(K, 2 * N + 1, dtype=dtype)[:, 1 : 2 * N + 1 : 2]
        b.copy_(w.t())
    exp = O.gemm_fxp(a, b, f, bits)
    bd = b.cuda() if layout != "kcontig" else w.cuda().t()
    if layout == "generic":
        bd = torch.zeros(K, 2 * N + 1, dtype=dtype, device="cuda")[:, 1 : 2 * N + 1 : 2]
        bd.copy_(w.t())
    got = G.gemm_fxp(a.cuda(), bd, f, bits).cpu()
    assert torch.equal(got, exp), (M, K, N, dtype, bits, layout, (got - exp).abs().max())
    gi = G.gemm_fxp_int(a.cuda(), bd, f, bits).cpu().to(torch.int64)
    ei = O.gemm_fxp_int(a, b, f, bits)
    if bits == 16:
        gi = O.wrap_int(gi, 16)
    assert torch.equal(gi, ei)


@pytest.mark.parametrize("layout", ["ncontig", "kcontig", "generic"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bits", [16, 32, 64])
def test_gemm_shapes(layout, dtype, bits):
    for (M, K, N) in [(1, 64, 128), (5, 33, 7), (16, 300, 257), (17, 128, 130), (64, 1024, 384)]:
        _gemm_case(M, K, N, dtype, bits, layout, f=8 if bits == 16 else 16)


@pytest.mark.parametrize("bits", [16, 32, 64])
def test_gemm_slow_path_saturation_nan(bits):
    """Large values fail the fast-path guard: exact clamp path, saturation, wrap."""
    for dtype in (torch.bfloat16, torch.float32):
        _gemm_case(33, 200, 130, dtype, bits, "ncontig", sa=300.0, sb=300.0, seed=3)
        _gemm_case(33, 200, 130, dtype, bits, "kcontig", sa=3000.0, sb=3000.0, seed=4)
    from fxpr_vllm.fixed_point_kernels import gemm as G

    a = torch.randn(4, 64)
    a[1, 3] = float("nan")
    a[2, 5] = float("inf")
    b = torch.randn(64, 140)
    got = G.gemm_fxp(a.cuda(), b.cuda(), 16, bits).cpu()
    assert torch.equal(got, O.gemm_fxp(a, b, 16, bits))


def test_gemm_decode_config_bitexact():
    """Full benchmark GEMM shape: A[64,4096] N(0,1) x W[4096,4096] N(0,0.02), bf16, Q15.16 int32."""
    _gemm_case(64, 4096, 4096, torch.bfloat16, 32, "ncontig", seed=0)


def test_gemm_k_permutation_and_determinism():
    from fxpr_vllm.fixed_point_kernels import gemm as G

    g = torch.Generator().manual_seed(123)
    a = torch.randn(4, 512, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(512, 256, generator=g).to(torch.bfloat16).cuda()
    perm = torch.randperm(512, generator=g).cuda()
    c0 = G.gemm_fxp(a, b, 16, 32)
    assert torch.equal(c0, G.gemm_fxp(a[:, perm], b[perm], 16, 32))
    for _ in range(3):
        assert torch.equal(c0, G.gemm_fxp(a, b, 16, 32))


def test_gemm_matches_float_matmul_tolerance():
    """Reference tests/test_gemm.py:25-55: close to torch.matmul (atol 5e-4)."""
    from fxpr_vllm.fixed_point_kernels import gemm as G

    g = torch.Generator(device="cuda").manual_seed(42)
    for (M, N, K) in [(4, 4, 16), (3, 7, 16), (1, 1, 32), (8, 16, 32)]:
        a = torch.randn(M, K, device="cuda", generator=g)
        b = torch.randn(K, N, device="cuda", generator=g)
        torch.testing.assert_close(G.gemm_fxp(a, b, 16, 32), a @ b, atol=5e-4, rtol=5e-4)
    eye = torch.eye(16, device="cuda")
    a = torch.randn(4, 16, device="cuda", generator=g)
    torch.testing.assert_close(G.gemm_fxp(a, eye, 16, 32), a, atol=1e-4, rtol=0)
    assert torch.equal(G.gemm_fxp(torch.ones(4, 16, device="cuda"), torch.zeros(16, 4, device="cuda"),
                                  16, 32), torch.zeros(4, 4, device="cuda"))


def test_gemm_empty_and_k0():
    from fxpr_vllm.fixed_point_kernels import gemm as G

    assert G.gemm_fxp(torch.zeros(0, 8, device="cuda"), torch.zeros(8, 5, device="cuda"), 16, 32).shape == (0, 5)
    out = G.gemm_fxp(torch.zeros(3, 0, device="cuda"), torch.zeros(0, 5, device="cuda"), 16, 32)
    assert torch.equal(out, torch.zeros(3, 5, device="cuda"))


def test_gemm_workspace_left_clean():
    from fxpr_vllm import _native as N
    from fxpr_vllm.fixed_point_kernels import gemm as G

    a = torch.randn(64, 4096, device="cuda").to(torch.bfloat16)
    b = torch.randn(4096, 512, device="cuda").to(torch.bfloat16)
    G.gemm_fxp(a, b, 16, 32)
    torch.cuda.synchronize()
    for key, buf in N._ws.items():
        if key[0] == "gemm":
            assert int(buf.count_nonzero()) == 0


# ------------------------------------------------- linear layer (GEMM + epilogue)
@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float32])
def test_linear_path_matches_oracle(bits, out_dtype, bias_dtype):
    """The path every model linear layer takes: fxpr::gemm_fxp_int (raw integer
    accumulator) then fxpr::fixed_to_float_bias (X2F + fp32 bias + cast),
    against the oracle's FixedPointLinearMethod.apply
    (reference vllm_modules/quantisation_config.py:163-187)."""
    from fxpr_vllm import library_ops  # noqa: F401

    g = torch.Generator().manual_seed(bits)
    f = 8 if bits == 16 else 16
    for (T, K, N) in [(1, 4096, 512), (7, 1000, 130), (64, 2048, 384)]:
        x = torch.randn(T, K, generator=g).to(out_dtype)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        bias = None if bias_dtype is None else torch.randn(N, generator=g).to(bias_dtype)
        acc = torch.ops.fxpr.gemm_fxp_int(x.cuda().to(torch.bfloat16), w.cuda().t(), f, bits)
        got = torch.ops.fxpr.fixed_to_float_bias(acc, None if bias is None else bias.cuda(), f, bits,
                                                 out_dtype).cpu()
        exp = O.linear_apply(x, w, bias, f, bits)
        assert got.dtype == out_dtype and bits_equal(got, exp), (T, K, N)


def test_linear_method_apply_matches_oracle():
    """FixedPointLinearMethod.apply itself (3-D activations, bias)."""
    from types import SimpleNamespace

    from fxpr_vllm.vllm_modules.quantisation_config import FixedPointConfig, FixedPointLinearMethod

    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 5, 1024, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, 1024, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.randn(256, generator=g).to(torch.bfloat16)
    m = FixedPointLinearMethod(FixedPointConfig(16))
    wd = w.cuda()
    layer = SimpleNamespace(weight_t=wd.t(), fxp_weight=wd, bias=None, fxp_int_reduce=False)
    got = m.apply(layer, x.cuda(), bias.cuda()).cpu()
    assert bits_equal(got, O.linear_apply(x, w, bias, 16, m.fxp_int_bits))


def test_lm_head_method_matches_oracle():
    """FixedPointLMHeadMethod.apply: logits of a vocabulary shard through the
    fixed-point GEMM, bf16 hidden states, with and without a bias."""
    from types import SimpleNamespace

    from fxpr_vllm.vllm_modules.quantisation_config import FixedPointConfig, FixedPointLMHeadMethod

    g = torch.Generator().manual_seed(9)
    x = torch.randn(5, 1024, generator=g).to(torch.bfloat16)
    w = (torch.randn(3000, 1024, generator=g) * 0.02).to(torch.bfloat16)
    m = FixedPointLMHeadMethod(FixedPointConfig(16))
    layer = SimpleNamespace(weight=w.cuda())
    for bias in (None, torch.randn(3000, generator=g).to(torch.bfloat16)):
        got = m.apply(layer, x.cuda(), None if bias is None else bias.cuda()).cpu()
        assert bits_equal(got, O.linear_apply(x, w, bias, 16, m.fxp_int_bits))
