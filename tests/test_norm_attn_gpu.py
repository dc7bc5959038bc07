"""RMSNorm, attention and log-softmax kernels against the oracle (bit-exact,
with the library's device primitives injected into the oracle)."""

import os

import pytest
import torch

from oracle import fxp_oracle as O
from tests.helpers import bits_equal, device_prims, paged_inputs

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def prims():
    return device_prims()


# ------------------------------------------------------------------- RMSNorm
def test_rms_norm_golden(prims):
    from fxpr_vllm.fixed_point_kernels import rms_norm as R

    for c in torch.load(os.path.join(GOLD, "rms_norm.pt"), weights_only=False):
        res = c["residual"].clone().cuda() if c["residual"] is not None else None
        y = R.rms_norm_fxp(c["x"].cuda(), c["w"].cuda(), c["eps"], c["frac"], c["bits"], residual=res).cpu()
        r = O.rms_norm_fxp(c["x"], c["w"], c["eps"], c["frac"], c["bits"], residual=c["residual"], prims=prims)
        if res is not None:
            assert torch.equal(res.cpu(), r[1]) and torch.equal(res.cpu(), c["residual_out"])
            r = r[0]
        assert bits_equal(y, r)
        # against the reference kernel's interpreter output (IEEE div/sqrt): a few ulp
        torch.testing.assert_close(y, c["out"], atol=0, rtol=4e-7)


@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm_random(prims, bits, dtype):
    from fxpr_vllm.fixed_point_kernels import rms_norm as R

    g = torch.Generator().manual_seed(bits)
    for (rows, hidden) in [(3, 7), (5, 4096), (2, 4100), (4, 13824)]:
        x = (torch.randn(rows, hidden, generator=g) * 2).to(dtype)
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
        r = (torch.randn(rows, hidden, generator=g)).to(dtype)
        f = 8 if bits == 16 else 16
        y = R.rms_norm_fxp(x.cuda(), w.cuda(), 1e-6, f, bits).cpu()
        assert bits_equal(y, O.rms_norm_fxp(x, w, 1e-6, f, bits, prims=prims))
        rd = r.cuda()
        y2 = R.rms_norm_fxp(x.cuda(), w.cuda(), 1e-5, f, bits, residual=rd).cpu()
        ey, er = O.rms_norm_fxp(x, w, 1e-5, f, bits, residual=r, prims=prims)
        assert bits_equal(y2, ey) and bits_equal(rd.cpu(), er)


def test_rms_norm_row_permutation():
    """Reference tests/test_rms_norm.py:115-135."""
    from fxpr_vllm.fixed_point_kernels import rms_norm as R

    xa = torch.tensor([64.0, 1.0, 1.0, 1.0, 1.0], device="cuda")
    perm = torch.tensor([1, 2, 3, 4, 0], device="cuda")
    x = torch.stack([xa, xa[perm]])
    y = R.rms_norm_fxp(x, torch.ones(5, device="cuda"), 1e-6, 16, 64)
    assert torch.equal(y[1], y[0][perm])


def test_rms_norm_config2_bitexact(prims):
    """Full benchmark RMSNorm shape: x[8192,4096] bf16 N(0,1), w N(1,0.1), eps 1e-6, int32 and int64."""
    from fxpr_vllm.fixed_point_kernels import rms_norm as R
    from fxpr_vllm.fixed_point_kernels import fixed_point as F

    g = torch.Generator().manual_seed(1)
    x = torch.randn(8192, 4096, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    for bits in (32, 64):
        y = R.rms_norm_fxp(x.cuda(), w.cuda(), 1e-6, 16, bits).cpu()
        assert bits_equal(y, O.rms_norm_fxp(x, w, 1e-6, 16, bits, prims=prims))
    assert torch.equal(F.fxp_sum(x.cuda(), 16, 32).cpu(), O.fxp_sum(x, 16, 32))


# ----------------------------------------------------------------- attention
def _run_attn(q, kv, qsl, sl, bt, max_q, **kw):
    """Both device paths (chunked with workspace, cluster without): identical bits."""
    from fxpr_vllm.fixed_point_kernels import attention as A

    outs = []
    for ws in (True, False):
        o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
        A.unified_attention_fxp(q.cuda(), kv.cuda(), o, qsl.cuda(), sl.cuda(), bt.cuda(), max_q,
                                use_workspace=ws, **kw)
        outs.append(o.cpu())
    assert bits_equal(outs[0], outs[1]), "chunked and cluster paths differ"
    return outs[0]


def _oracle_attn(q, kv, qsl, sl, bt, max_q, prims, bits=32, **kw):
    o = torch.zeros(q.shape, dtype=torch.float32)
    return O.unified_attention_fxp(q, kv, o, qsl, sl, bt, max_q, int_bits=bits, prims=prims, **kw)


def test_attention_golden(prims):
    for c in torch.load(os.path.join(GOLD, "attention.pt"), weights_only=False):
        slopes = c["alibi_slopes"] * O.RCP_LN2 if c["alibi_slopes"] is not None else None
        kw = dict(is_causal=c["causal"], frac_bits=c["frac"], logits_soft_cap=c["softcap"],
                  window_size=c["window"])
        got = _run_attn(c["q"], c["kv_cache"], c["query_start_loc"], c["seq_lens"], c["block_table"],
                        c["max_query_len"], alibi_slopes=slopes.cuda() if slopes is not None else None,
                        fxp_dtype=c["bits"], **kw)
        exp = _oracle_attn(c["q"], c["kv_cache"], c["query_start_loc"], c["seq_lens"],
                           c["block_table"], c["max_query_len"], prims, bits=c["bits"],
                           alibi_slopes=slopes, **kw)
        assert bits_equal(got, exp), (c["seq_lens"], (got - exp).abs().max())
        torch.testing.assert_close(got, c["out"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("bits", [32, 64])
@pytest.mark.parametrize("D", [64, 128])
def test_attention_decode_gqa(prims, bits, D):
    q, kv, qsl, sl, bt = paged_inputs([1] * 5, [1, 17, 200, 513, 700], 8, 2, D, 16, seed=D)
    exp = _oracle_attn(q, kv, qsl, sl, bt, 1, prims, bits=bits, frac_bits=16)
    for splits in (1, 3, 8, 16):
        got = _run_attn(q, kv, qsl, sl, bt, 1, fxp_dtype=bits, frac_bits=16, num_kv_splits=splits)
        assert bits_equal(got, exp), (splits, (got - exp).abs().max())


def test_attention_prefill_chunked(prims):
    q, kv, qsl, sl, bt = paged_inputs([70, 1, 9], [100, 33, 9], 4, 2, 128, 16, seed=5)
    exp = _oracle_attn(q, kv, qsl, sl, bt, 70, prims, frac_bits=16)
    for splits in (1, 4):
        got = _run_attn(q, kv, qsl, sl, bt, 70, frac_bits=16, num_kv_splits=splits)
        assert bits_equal(got, exp)


def test_attention_fp32_inputs_page1(prims):
    """The reference's prefill tests use fp32 q/k/v and a page_size=1 cache."""
    q, kv, qsl, sl, bt = paged_inputs([32, 32], [32, 32], 2, 2, 32, 1, dtype=torch.float32, seed=7)
    for causal in (True, False):
        exp = _oracle_attn(q, kv, qsl, sl, bt, 32, prims, frac_bits=14, is_causal=causal)
        got = _run_attn(q, kv, qsl, sl, bt, 32, frac_bits=14, is_causal=causal)
        assert bits_equal(got, exp)


def test_attention_large_values_slow_path(prims):
    q, kv, qsl, sl, bt = paged_inputs([1, 2], [50, 90], 4, 1, 64, 16, seed=9)
    kv = kv * 300  # fails the magic-constant guards: exact path
    q = q * 30
    exp = _oracle_attn(q, kv, qsl, sl, bt, 2, prims, frac_bits=16)
    got = _run_attn(q, kv, qsl, sl, bt, 2, frac_bits=16)
    assert bits_equal(got, exp)


def test_attention_long_context_rescore(prims):
    """Keys beyond the score capacity of one CTA are re-scored in pass 2."""
    q, kv, qsl, sl, bt = paged_inputs([1], [20000], 4, 1, 128, 16, seed=11)
    exp = _oracle_attn(q, kv, qsl, sl, bt, 1, prims, frac_bits=16)
    got = _run_attn(q, kv, qsl, sl, bt, 1, frac_bits=16, num_kv_splits=1)
    assert bits_equal(got, exp)
    got8 = _run_attn(q, kv, qsl, sl, bt, 1, frac_bits=16, num_kv_splits=8)
    assert bits_equal(got8, exp)


@pytest.mark.parametrize("bits", [32, 64])
def test_attention_chunk_boundaries(prims, bits):
    """Context lengths around the 512-key work units of the chunked path,
    ragged batch, decode and short prefill rows; the workspace is filled with
    garbage between calls (it carries no state)."""
    from fxpr_vllm import _native as N

    lens = [1, 511, 512, 513, 1023, 1024, 1025, 3000]
    q, kv, qsl, sl, bt = paged_inputs([1] * len(lens), lens, 8, 2, 128, 16, seed=21)
    exp = _oracle_attn(q, kv, qsl, sl, bt, 1, prims, bits=bits, frac_bits=16)
    for _ in range(3):
        got = _run_attn(q, kv, qsl, sl, bt, 1, fxp_dtype=bits, frac_bits=16)
        assert bits_equal(got, exp), (got - exp).abs().max()
        for key, buf in N._ws.items():
            if key[0] == "attn":
                buf.random_(0, 256)
    q, kv, qsl, sl, bt = paged_inputs([5, 1, 17], [1030, 513, 600], 8, 2, 64, 16, seed=22)
    exp = _oracle_attn(q, kv, qsl, sl, bt, 17, prims, bits=bits, frac_bits=16)
    got = _run_attn(q, kv, qsl, sl, bt, 17, fxp_dtype=bits, frac_bits=16)
    assert bits_equal(got, exp), (got - exp).abs().max()


def test_attention_decode_large_values_rq(prims):
    """Decode (4-row) scores kernel: lanes on the exact path next to fast ones,
    64-bit and 32-bit accumulators, several chunks."""
    q, kv, qsl, sl, bt = paged_inputs([1] * 3, [700, 90, 1500], 8, 2, 128, 16, seed=23)
    kv = kv.clone()
    kv[::7] *= 300  # some pages fail the magic-constant guard
    q = q * 30
    for bits in (32, 64):
        exp = _oracle_attn(q, kv, qsl, sl, bt, 1, prims, bits=bits, frac_bits=16)
        got = _run_attn(q, kv, qsl, sl, bt, 1, fxp_dtype=bits, frac_bits=16)
        assert bits_equal(got, exp), (bits, (got - exp).abs().max())


def test_attention_kv_permutation_invariance():
    """Reference tests/test_prefill.py:232-275 (non-causal, permuted keys)."""
    q, kv, qsl, sl, bt = paged_inputs([32], [32], 2, 2, 32, 1, dtype=torch.float32, seed=3)
    o1 = _run_attn(q, kv, qsl, sl, bt, 32, frac_bits=14, is_causal=False)
    perm = torch.randperm(32)
    kv2 = kv.clone()
    kv2[bt[0, :32].long()] = kv[bt[0, perm].long()]
    o2 = _run_attn(q, kv2, qsl, sl, bt, 32, frac_bits=14, is_causal=False)
    assert torch.equal(o1, o2)


def test_attention_bf16_output_and_tolerance():
    """Close to float softmax attention (reference tests/test_prefill.py atol 5e-2)."""
    q, kv, qsl, sl, bt = paged_inputs([1, 1], [300, 40], 8, 2, 128, 16, seed=2)
    from fxpr_vllm.fixed_point_kernels import attention as A

    o = torch.zeros(q.shape, dtype=torch.bfloat16, device="cuda")
    A.unified_attention_fxp(q.cuda(), kv.cuda(), o, qsl.cuda(), sl.cuda(), bt.cuda(), 1, frac_bits=16)
    for r in range(2):
        L = int(sl[r])
        keys = torch.arange(L)
        blk, slot = bt[r, keys // 16].long(), keys % 16
        for h in range(8):
            k = kv[blk, 0, slot, h // 4].float()
            v = kv[blk, 1, slot, h // 4].float()
            p = torch.softmax((q[r, h].float() @ k.T) / 128**0.5, -1)
            torch.testing.assert_close(o[r, h].float().cpu(), p @ v, atol=5e-2, rtol=5e-2)


# --------------------------------------------------------------- log-softmax
def test_log_softmax(prims):
    from fxpr_vllm.fixed_point_kernels import softmax as S

    for c in torch.load(os.path.join(GOLD, "log_softmax.pt"), weights_only=False):
        got = S.log_softmax_fxp(c["x"].cuda(), c["bits"], frac_bits=c["frac"]).cpu()
        assert bits_equal(got, O.log_softmax_fxp(c["x"], c["bits"], c["frac"], prims=prims))
        torch.testing.assert_close(got, c["out"], atol=1e-5, rtol=1e-5)


def test_workspace_growth_keeps_captured_graph_valid():
    """A CUDA graph records the workspace address of the call it captured. A
    later eager call that needs a larger workspace must not free that buffer:
    replaying the graph afterwards still gives the captured call's result,
    and the eager call's own result is unaffected."""
    from fxpr_vllm.fixed_point_kernels import attention as A
    from fxpr_vllm.fixed_point_kernels import gemm as G

    q, kv, qsl, sl, bt = paged_inputs([1] * 3, [600, 90, 1100], 8, 2, 128, 16, seed=31)
    dq, dkv, dqsl, dsl, dbt = (t.cuda() for t in (q, kv, qsl, sl, bt))
    a = torch.randn(16, 2048, device="cuda").to(torch.bfloat16)
    b = torch.randn(2048, 256, device="cuda").to(torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
        A.unified_attention_fxp(dq, dkv, o, dqsl, dsl, dbt, 1, frac_bits=16)  # warm-up, sizes the buffers
        c = G.gemm_fxp(a, b, 16, 32)
        torch.cuda.synchronize()
        expect_o, expect_c = o.clone(), c.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            o.zero_()
            A.unified_attention_fxp(dq, dkv, o, dqsl, dsl, dbt, 1, frac_bits=16)
            c2 = G.gemm_fxp(a, b, 16, 32)
        # eager calls on the same stream that need far larger workspaces
        q3, kv3, qsl3, sl3, bt3 = paged_inputs([1] * 40, [3000] * 40, 8, 2, 128, 16, seed=32)
        o3 = torch.zeros(q3.shape, dtype=torch.float32, device="cuda")
        A.unified_attention_fxp(q3.cuda(), kv3.cuda(), o3, qsl3.cuda(), sl3.cuda(), bt3.cuda(), 1,
                                frac_bits=16)
        big = G.gemm_fxp(torch.randn(64, 8192, device="cuda").to(torch.bfloat16),
                         torch.randn(8192, 1024, device="cuda").to(torch.bfloat16), 16, 32)
        junk = torch.empty(64 << 20, dtype=torch.uint8, device="cuda").fill_(0xAB)  # reuse freed memory
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
    assert bits_equal(o, expect_o) and bits_equal(c2, expect_c)
    del junk, big


def test_attention_understated_hint(monkeypatch, prims):
    """A max_seq_len hint below a context length: with FXPR_VALIDATE_HINTS=1
    the call raises; without it the kernels stay inside the workspace sized
    from the hint (no overrun) and the other requests are still exact."""
    from fxpr_vllm.fixed_point_kernels import attention as A

    q, kv, qsl, sl, bt = paged_inputs([1, 1], [300, 2000], 8, 2, 128, 16, seed=41)
    o = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    args = (q.cuda(), kv.cuda(), o, qsl.cuda(), sl.cuda(), bt.cuda(), 1)
    monkeypatch.setenv("FXPR_VALIDATE_HINTS", "1")
    with pytest.raises(ValueError, match="max_seq_len"):
        A.unified_attention_fxp(*args, frac_bits=16, max_seq_len=1000)
    monkeypatch.setenv("FXPR_VALIDATE_HINTS", "0")
    A.unified_attention_fxp(*args, frac_bits=16, max_seq_len=1000)
    torch.cuda.synchronize()
    exp = _oracle_attn(q[:1], kv, qsl[:2], sl[:1], bt[:1], 1, prims, frac_bits=16)
    assert bits_equal(o[:1].cpu(), exp)


@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fixed_to_float_add_rms_norm(prims, bits, dtype):
    """The fused row-parallel epilogue + residual RMSNorm against the oracle
    composition (linear epilogue, quantisation_config.py:181-187, then
    rms_norm.py:36-59) and against the two unfused device ops."""
    from fxpr_vllm import library_ops  # noqa: F401

    g = torch.Generator().manual_seed(bits)
    f = 8 if bits == 16 else 16
    for rows, hidden in [(3, 4096), (7, 1000)]:
        lim = 2 ** (15 if bits == 16 else 30)
        acc = torch.randint(-lim, lim, (rows, hidden), generator=g,
                            dtype=torch.int64 if bits == 64 else torch.int32)
        bias = torch.randn(hidden, generator=g).to(dtype)
        res = torch.randn(rows, hidden, generator=g).to(dtype)
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
        for b in (None, bias):
            rd = res.clone().cuda()
            y = torch.ops.fxpr.fixed_to_float_add_rms_norm(acc.cuda(), None if b is None else b.cuda(), rd,
                                                           w.cuda(), 1e-5, f, bits)
            # oracle: X2F + bias in fp32, cast to the activation dtype, residual RMSNorm
            a = acc if bits != 16 else O.wrap_int(acc.to(torch.int64), 16)
            h = O.fixed_to_float(a, f, torch.float32)
            if b is not None:
                h = h + b.to(torch.float32)
            ey, er = O.rms_norm_fxp(h.to(dtype), w, 1e-5, f, bits, residual=res, prims=prims)
            assert bits_equal(y.cpu(), ey) and bits_equal(rd.cpu(), er), (rows, hidden, b is None)
            # the unfused pair on the device
            r2 = res.clone().cuda()
            h2 = torch.ops.fxpr.fixed_to_float_bias(acc.cuda(), None if b is None else b.cuda(), f, bits, dtype)
            y2 = torch.ops.fxpr.rms_norm_fxp_residual(h2, r2, w.cuda(), 1e-5, f, bits)
            assert bits_equal(y, y2) and bits_equal(rd, r2)
