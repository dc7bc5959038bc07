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
from oracle import fxp_oracle as O

pytestmark = pytest.mark.gpu

SCRATCH = 8 << 20  # bytes of the library's fixed scratch array


def _noalloc(a, b, frac, bits):
    c = torch.empty(a.shape[0], b.shape[1], dtype=torch.float32, device=a.device)
    rc = N.load().fxpr_gemm_fxp_noalloc(
        a.data_ptr(), N.dcode(a), a.stride(0), a.stride(1), b.data_ptr(), N.dcode(b),
        b.stride(0), b.stride(1), c.data_ptr(), 0, c.stride(0), c.stride(1),
        a.shape[0], b.shape[1], a.shape[1], frac, bits, N.stream_ptr(a.device))
    N.check(rc, "gemm_fxp_noalloc")
    return c


@pytest.mark.parametrize("bits", [32, 64])
def test_noalloc_matches_workspace_entry_and_oracle_twice(bits):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    w = (torch.randn(1024, 4096, generator=g) * 0.02).to(torch.bfloat16)
    assert N.load().fxpr_gemm_workspace_bytes(64, 1024, 4096, bits) > 0  # uses the scratch
    exp = O.gemm_fxp(a, w.t(), 16, bits)
    ad, wd = a.cuda(), w.cuda()
    ref = G.gemm_fxp(ad, wd.t(), 16, bits)
    for _ in range(2):  # the second call sees the first call's leftover scratch
        got = _noalloc(ad, wd.t(), 16, bits)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
        assert torch.equal(got.cpu(), exp)


def test_noalloc_rejects_shapes_beyond_the_scratch():
    lib = N.load()
    M, K = 64, 4096
    # split-K (and so the scratch) is used while the output tiles do not fill
    # the GPU; find a width whose int64 partials need more than the fixed array
    widths = [128 * t for t in range(1, 4096)
              if lib.fxpr_gemm_workspace_bytes(M, 128 * t, K, 64) > SCRATCH]
    if not widths:
        # split-K is only used while the output tiles fill less than the GPU, so
        # the scratch is bounded by about (SMs x 32 KB); on a 148-SM B200 that
        # is ~4.8 MB and every shape fits the array
        pytest.skip("no shape on this GPU needs more split-K scratch than the fixed array "
                    f"({lib.fxpr_gemm_workspace_bytes(M, 128 * 147, K, 64)} bytes at most here)")
    N_ = widths[0]
    a = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(K, N_, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(a, b, 16, 64)
