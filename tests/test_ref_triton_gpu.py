"""The CUDA kernels against the reference plugin's own Triton kernels, as
Triton 3.6 lowers them for B200 and run on the same device: bit for bit.

This pins what the CPU oracle cannot: the reference's floating-point steps
whose rounding is the GPU compiler's choice -- exp2, the fast divide and
square root, and any multiply-add contraction Triton applies around them
(`qk * scale - max` before exp2, the ALiBi term, the softcap, `1/sqrt`).
The reference kernels are compiled ahead of time from the reference
checkout by oracle/build_ref.py into oracle/_ref/ and launched through
oracle/ref_triton.py (fixed_point_kernels/attention.py:282-489,
rms_norm.py:10-60, gemm.py:134-196, softmax.py:8-97).
"""

import pytest
import torch

import bench
from oracle import ref_triton as RT
from tests.helpers import bits_equal, paged_inputs

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not RT.available("attn_d128_g4_i32"),
                       reason="reference kernels not built (python oracle/build_ref.py)"),
]

RCP_LN2 = 1.4426950408889634


def _ours(q, kv, qsl, sl, bt, max_q, bits, **kw):
    from fxpr_vllm.fixed_point_kernels import attention as A

    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    A.unified_attention_fxp(q, kv, o, qsl, sl, bt, max_q, fxp_dtype=bits, frac_bits=16, **kw)
    return o


def _ref(name, q, kv, qsl, sl, bt, max_q, alibi=None, softmax_scale=None):
    from fxpr_vllm.fixed_point_kernels import attention as A

    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    scale = A.prepare_log2_softmax_scale(q.shape[-1], softmax_scale)
    RT.attention(name, q, kv, o, qsl, sl, bt, max_q, scale, alibi_slopes=alibi)
    return o


def _diff(a, b):
    d = (a.view(torch.int32) != b.view(torch.int32))
    return f"{int(d.sum())} of {d.numel()} differ, max abs {float((a - b).abs().max()):.3g}"


@pytest.mark.parametrize("D,bits", [(128, 32), (128, 64), (64, 32)])
def test_attention_decode_vs_reference_kernel(D, bits):
    q, kv, qsl, sl, bt = (t.cuda() for t in paged_inputs([1] * 6, [1, 17, 200, 513, 700, 2100],
                                                         8, 2, D, 16, seed=D + bits))
    got = _ours(q, kv, qsl, sl, bt, 1, bits)
    exp = _ref(f"attn_d{D}_g4_i{bits}", q, kv, qsl, sl, bt, 1)
    assert bits_equal(got, exp), _diff(got, exp)


@pytest.mark.parametrize("bits", [32, 64])
def test_attention_config3_vs_reference_kernel(bits):
    """All 64 requests of the decode-attention benchmark shape."""
    d = {k: v.cuda() for k, v in bench.attention_inputs(seed=2).items()}
    got = _ours(d["Q"], d["KV"], d["qsl"], d["seq_lens"], d["bt"], 1, bits, max_seq_len=8192)
    exp = _ref(f"attn_d128_g4_i{bits}", d["Q"], d["KV"], d["qsl"], d["seq_lens"], d["bt"], 1)
    assert bits_equal(got, exp), _diff(got, exp)


def test_attention_prefill_vs_reference_kernel():
    q, kv, qsl, sl, bt = (t.cuda() for t in paged_inputs([70, 1, 9, 130], [100, 33, 9, 300], 8, 2, 128,
                                                         16, seed=5))
    got = _ours(q, kv, qsl, sl, bt, 130, 32)
    exp = _ref("attn_d128_g4_i32", q, kv, qsl, sl, bt, 130)
    assert bits_equal(got, exp), _diff(got, exp)


def test_attention_alibi_softcap_window_vs_reference_kernel():
    q, kv, qsl, sl, bt = (t.cuda() for t in paged_inputs([1, 5, 1], [300, 260, 40], 8, 2, 128, 16,
                                                         seed=9))
    g = torch.Generator().manual_seed(3)
    slopes = (torch.rand(8, generator=g) * 0.5).to(torch.float32) * RCP_LN2
    slopes = slopes.cuda()
    got = _ours(q, kv, qsl, sl, bt, 5, 32, alibi_slopes=slopes)
    exp = _ref("attn_d128_g4_i32_alibi", q, kv, qsl, sl, bt, 5, alibi=slopes)
    assert bits_equal(got, exp), "alibi: " + _diff(got, exp)
    got = _ours(q, kv, qsl, sl, bt, 5, 32, logits_soft_cap=30.0)
    exp = _ref("attn_d128_g4_i32_softcap30", q, kv, qsl, sl, bt, 5)
    assert bits_equal(got, exp), "softcap: " + _diff(got, exp)
    got = _ours(q, kv, qsl, sl, bt, 5, 32, window_size=100)
    exp = _ref("attn_d128_g4_i32_window100", q, kv, qsl, sl, bt, 5)
    assert bits_equal(got, exp), "window: " + _diff(got, exp)


@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("residual", [False, True])
def test_rms_norm_vs_reference_kernel(bits, residual):
    """fp32 rows as the reference glue passes them, and the bf16 path against
    the reference's fp32 result cast back to bf16 (vllm_modules/rms_norm.py:62-99)."""
    from fxpr_vllm.fixed_point_kernels import rms_norm as R

    f = 8 if bits == 16 else 16
    g = torch.Generator().manual_seed(bits + 7 * residual)
    for eps in (1e-6, 1e-5):
        name = f"rms_h4096_i{bits}_r{int(residual)}_eps{eps:g}"
        x = (torch.randn(64, 4096, generator=g) * 2).cuda()
        w = (1 + 0.1 * torch.randn(4096, generator=g)).cuda()
        r = torch.randn(64, 4096, generator=g).cuda() if residual else None
        y_ref = torch.empty_like(x)
        r_ref = r.clone() if residual else None
        RT.rms_norm(name, x, w, y_ref, r_ref)
        r_ours = r.clone() if residual else None
        y = R.rms_norm_fxp(x, w, eps, f, bits, residual=r_ours)
        assert bits_equal(y, y_ref), f"eps={eps}: " + _diff(y, y_ref)
        if residual:
            assert bits_equal(r_ours, r_ref)
        # bf16 activations: the reference glue widens to fp32 and casts back
        xb, wb = x.to(torch.bfloat16), w.to(torch.bfloat16)
        y_ref = torch.empty_like(x)
        rb = r.to(torch.bfloat16) if residual else None
        r_ref = rb.float() if residual else None
        RT.rms_norm(name, xb.float(), wb.float(), y_ref, r_ref)
        rb_ours = rb.clone() if residual else None
        yb = R.rms_norm_fxp(xb, wb, eps, f, bits, residual=rb_ours)
        assert bits_equal(yb, y_ref.to(torch.bfloat16)), f"bf16 eps={eps}"
        if residual:
            assert bits_equal(rb_ours, r_ref.to(torch.bfloat16))


@pytest.mark.parametrize("bits", [32, 64])
def test_gemm_vs_reference_kernel(bits):
    from fxpr_vllm.fixed_point_kernels import gemm as G

    inp = bench.gemm_inputs(0)
    a = inp["A"].cuda()
    w = inp["W"].cuda()
    wt = w.t().contiguous()  # the reference linear method's weight_t (quantisation_config.py:157)
    c_ref = torch.empty(a.shape[0], wt.shape[1], dtype=torch.float32, device="cuda")
    RT.gemm(f"gemm_bf16_i{bits}", a, wt, c_ref)
    assert bits_equal(G.gemm_fxp(a, wt, 16, bits), c_ref)
    assert bits_equal(G.gemm_fxp(a, w.t(), 16, bits), c_ref)


@pytest.mark.parametrize("bits", [32, 64])
def test_log_softmax_vs_reference_kernel(bits):
    from fxpr_vllm.fixed_point_kernels import softmax as S

    g = torch.Generator().manual_seed(bits)
    x = (torch.randn(37, 1000, generator=g) * 4).cuda()
    y_ref = torch.empty_like(x)
    RT.log_softmax(f"log_softmax_n1024_i{bits}", x, y_ref)
    y = S.log_softmax_fxp(x, bits, frac_bits=16)
    assert bits_equal(y, y_ref), _diff(y, y_ref)
