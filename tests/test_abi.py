"""The C-ABI library loads and exports every symbol include/fxpr_b200.h
declares; argument validation runs on the host (no GPU needed)."""

import ctypes
import os
import re

import pytest
import torch

from fxpr_vllm import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "fxpr_b200.h")


def header_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(fxpr_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = N.load()
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(N.EXPORTED)


def test_abi_version():
    assert N.load().fxpr_abi_version() == 3


def test_invalid_bits_rejected_before_launch():
    lib = N.load()
    rc = lib.fxpr_float_to_fixed(None, N.F32, None, 24, 10, 16, None)
    assert rc == N.FXPR_ERR_INVALID
    assert "16/32/64" in lib.fxpr_last_error().decode()
    with pytest.raises(ValueError):
        N.check(rc, "float_to_fixed")


def test_gemm_rejects_missing_workspace():
    lib = N.load()
    need = lib.fxpr_gemm_workspace_bytes(64, 4096, 4096, 32)
    assert need > 0  # decode shapes use split-K
    rc = lib.fxpr_gemm_fxp(None, N.BF16, 4096, 1, None, N.BF16, 4096, 1, None, 0, 4096, 1,
                           64, 4096, 4096, 16, 32, None, 0, None)
    assert rc == N.FXPR_ERR_INVALID
    assert "workspace" in lib.fxpr_last_error().decode()


def test_gemm_bad_frac_bits():
    lib = N.load()
    rc = lib.fxpr_gemm_fxp(None, N.BF16, 1, 1, None, N.BF16, 1, 1, None, 0, 1, 1,
                           1, 1, 1, 200, 32, None, 0, None)
    assert rc == N.FXPR_ERR_INVALID


def test_attention_rejects_int16_and_bad_head_dim():
    lib = N.load()
    p = N.AttentionParams()
    p.int_bits = 16
    p.head_dim = 128
    assert lib.fxpr_unified_attention_fxp(ctypes.byref(p), None) == N.FXPR_ERR_UNSUPPORTED
    p.int_bits = 32
    p.head_dim = 100
    assert lib.fxpr_unified_attention_fxp(ctypes.byref(p), None) == N.FXPR_ERR_UNSUPPORTED


def test_cpu_tensors_fail_loudly():
    from fxpr_vllm.fixed_point_kernels import gemm

    with pytest.raises(RuntimeError, match="CUDA"):
        gemm.gemm_fxp(torch.zeros(2, 3), torch.zeros(3, 4), 16, 32)


def test_library_ops_have_no_cpu_kernel():
    import fxpr_vllm.library_ops  # noqa: F401

    with pytest.raises(Exception):
        torch.ops.fxpr.gemm_fxp(torch.zeros(2, 3), torch.zeros(3, 4), 16, 32)


def test_fake_impls_shape():
    import fxpr_vllm.library_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = torch.empty(5, 7, device="cuda") if torch.cuda.is_available() else torch.empty(5, 7)
        b = torch.empty(7, 3, device=a.device)
        c = torch.ops.fxpr.gemm_fxp(a, b, 16, 32)
        assert c.shape == (5, 3) and c.dtype == torch.float32
        ci = torch.ops.fxpr.gemm_fxp_int(a, b, 16, 64)
        assert ci.dtype == torch.int64


def test_attention_workspace_query():
    """The workspace query: 0 for shapes the chunked path does not take."""
    p = N.AttentionParams()
    p.num_requests, p.max_query_len, p.num_heads, p.num_kv_heads = 64, 1, 32, 8
    p.head_dim, p.page_size, p.max_seq_len, p.int_bits = 128, 16, 8192, 32
    p.q_dtype = p.kv_dtype = p.o_dtype = 1
    need = N.load().fxpr_attention_workspace_bytes(ctypes.byref(p))
    assert need >= 64 * 8 * 16 * 4 * 512 * 4  # scores of every (item, chunk, row, key)
    p.max_seq_len = 1 << 24  # scratch beyond the limit: cluster path
    assert N.load().fxpr_attention_workspace_bytes(ctypes.byref(p)) == 0
    p.max_seq_len, p.int_bits = 8192, 16  # invalid: 0
    assert N.load().fxpr_attention_workspace_bytes(ctypes.byref(p)) == 0



def test_attention_max_seq_len_hint_check():
    """An understated max_seq_len hint is reported instead of silently
    cutting the context (the check FXPR_VALIDATE_HINTS=1 runs before launch)."""
    from fxpr_vllm.fixed_point_kernels import attention as A

    sl = torch.tensor([100, 900], dtype=torch.int32)
    A.check_max_seq_len_hint(sl, 900)
    A.check_max_seq_len_hint(sl[:0], 1)
    with pytest.raises(ValueError, match="max_seq_len=512"):
        A.check_max_seq_len_hint(sl, 512)
