"""The allocation-free GEMM entry point (fxpr_gemm_fxp_noalloc).

It exists for callers that cannot allocate device memory while they run --
e.g. an engine whose device memory is planned once up front, or a binding
from another language with no device allocator -- and keeps its split-K
scratch in a fixed array inside the library. This file is collected last so
that a run stopping at the first failure has run every other test already.
"""

import pytest
import torch

from fxpr_vllm import _native as N
from fxpr_vllm.fixed_point_kernels import gemm as G

pytestmark = pytest.mark.gpu


def _noalloc(a, b, frac, bits):
    c = torch.empty(a.shape[0], b.shape[1], dtype=torch.float32, device=a.device)
    rc = N.load().fxpr_gemm_fxp_noalloc(
        a.data_ptr(), N.dcode(a), a.stride(0), a.stride(1), b.data_ptr(), N.dcode(b),
        b.stride(0), b.stride(1), c.data_ptr(), 0, c.stride(0), c.stride(1),
        a.shape[0], b.shape[1], a.shape[1], frac, bits, N.stream_ptr(a.device))
    N.check(rc, "gemm_fxp_noalloc")
    return c


@pytest.mark.parametrize("bits", [32, 64])
def test_noalloc_matches_workspace_entry_twice(bits):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(64, 4096, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(1024, 4096, generator=g) * 0.02).to(torch.bfloat16).cuda()
    assert N.load().fxpr_gemm_workspace_bytes(64, 1024, 4096, bits) > 0  # uses the scratch
    ref = G.gemm_fxp(a, w.t(), 16, bits)
    for _ in range(2):  # the second call sees the first call's leftover scratch
        got = _noalloc(a, w.t(), 16, bits)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


def test_noalloc_rejects_shapes_beyond_the_scratch():
    # 140 output tiles with split-K and int64 partials need ~9.2 MB > 8 MiB
    M, N, K = 64, 140 * 128, 4096
    need = N_lib().fxpr_gemm_workspace_bytes(M, N, K, 64)
    if need <= 8 << 20:
        pytest.skip("shape does not need more than the fixed scratch on this device")
    a = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(K, N, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(a, b, 16, 64)


def N_lib():
    return N.load()
