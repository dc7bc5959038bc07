"""Generate golden vectors from the reference's own Triton kernels.

Runs in the build container only (it imports the reference project, which is
not present on the GPU box): the reference kernels execute on the Triton CPU
interpreter (``TRITON_INTERPRET=1``). Interpreter gaps that are bridged:

* ``libdevice.rint`` / ``libdevice.tanh`` are not implemented by the
  interpreter; they are replaced with numpy ``rint`` / ``tanh`` (rint is
  exact, so this changes nothing for the casts).
* the interpreter truncates fp32 -> bf16 stores, the GPU rounds; all output
  buffers are therefore fp32.
* the interpreter cannot wrap an int32 reduction (it raises), so the
  RMSNorm cases keep the squared-sum inside int32.

Usage:  python tests/golden/make_golden.py /path/to/reference
Writes ``tests/golden/*.pt`` (inputs + reference outputs, small shapes).
"""

from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

OUT_DIR = os.path.dirname(os.path.abspath(__file__))

FP = None  # the reference's fixed_point module, bound in main()


def _patch_libdevice():
    from triton.runtime.interpreter import TensorHandle
    import triton.language.extra.libdevice as ld
    import triton.language.extra.cuda.libdevice as cld

    def _wrap(fn):
        def f(x, _semantic=None):
            data = fn(x.handle.data)
            return tl.tensor(TensorHandle(data.astype(x.handle.data.dtype), x.handle.dtype), x.type)

        return f

    for mod in (ld, cld):
        mod.rint = _wrap(np.rint)
        mod.tanh = _wrap(np.tanh)


@triton.jit
def _f2x(x_ptr, y_ptr, n, F: tl.constexpr, BLOCK: tl.constexpr, OUT: tl.constexpr):
    offs = tl.arange(0, BLOCK)
    m = offs < n
    tl.store(y_ptr + offs, FP.float_to_fixed(tl.load(x_ptr + offs, mask=m), F, OUT), mask=m)


@triton.jit
def _x2f(x_ptr, y_ptr, n, F: tl.constexpr, BLOCK: tl.constexpr, OUT: tl.constexpr):
    offs = tl.arange(0, BLOCK)
    m = offs < n
    tl.store(y_ptr + offs, FP.fixed_to_float(tl.load(x_ptr + offs, mask=m), F, OUT), mask=m)


def main(ref_root: str) -> None:
    global FP
    sys.path.insert(0, ref_root)
    _patch_libdevice()
    from fxpr_vllm.fixed_point_kernels import fixed_point as _fp

    FP = _fp
    from fxpr_vllm.fixed_point_kernels import gemm as G
    from fxpr_vllm.fixed_point_kernels import rms_norm as RN
    from fxpr_vllm.fixed_point_kernels import attention as AT
    from fxpr_vllm.fixed_point_kernels import softmax as SM

    TL_INT = {16: tl.int16, 32: tl.int32, 64: tl.int64}
    T_INT = {16: torch.int16, 32: torch.int32, 64: torch.int64}
    TL_F = {torch.float32: tl.float32, torch.float64: tl.float64}

    g = torch.Generator().manual_seed(1234)

    # ---------------- casts ----------------
    casts = []
    base = torch.cat([
        torch.tensor([0.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.49999, 1e30, -1e30, 7.0, -7.0]),
        torch.randn(200, generator=g) * 4,
        torch.randn(50, generator=g) * 1e5,
        (torch.randint(-4096, 4096, (50,), generator=g).float() + 0.5) / 16,  # exact ties at f=4
    ])
    for fdt in (torch.float32, torch.float64):
        x = base.to(fdt)
        for bits in (16, 32, 64):
            for f in (0, 4, 14, 16):
                n = x.numel()
                y = torch.empty(n, dtype=T_INT[bits])
                _f2x[(1,)](x, y, n, F=f, BLOCK=triton.next_power_of_2(n), OUT=TL_INT[bits])
                casts.append(dict(kind="f2x", x=x.clone(), frac=f, bits=bits, out=y.clone()))
    for bits in (32, 64):
        q = torch.randint(-(2**31), 2**31 - 1, (300,), generator=g).to(T_INT[bits])
        if bits == 64:
            q = q * 1234567
        for f in (0, 8, 16):
            for fdt in (torch.float32, torch.float64):
                n = q.numel()
                y = torch.empty(n, dtype=fdt)
                _x2f[(1,)](q, y, n, F=f, BLOCK=triton.next_power_of_2(n), OUT=TL_F[fdt])
                casts.append(dict(kind="x2f", x=q.clone(), frac=f, bits=bits, fdt=str(fdt), out=y.clone()))
    torch.save(casts, os.path.join(OUT_DIR, "casts.pt"))
    print("casts", len(casts))

    # ---------------- GEMM ----------------
    gemms = []
    cases = [
        (5, 40, 7, torch.bfloat16, 1.0, 0.02, 16, 32),
        (3, 70, 9, torch.float32, 1.0, 1.0, 16, 32),
        (4, 33, 6, torch.bfloat16, 1.0, 0.5, 8, 16),
        (6, 64, 5, torch.bfloat16, 1.0, 0.02, 16, 64),
        (2, 50, 3, torch.bfloat16, 300.0, 300.0, 16, 32),  # per-product saturation + wrap
        (3, 20, 4, torch.float32, 3000.0, 3000.0, 0, 16),  # int16 saturation + wrap
        (7, 129, 65, torch.float16, 1.0, 0.1, 14, 32),
    ]
    for (M, K, N, dt, sa, sb, f, bits) in cases:
        a = (torch.randn(M, K, generator=g) * sa).to(dt)
        b = (torch.randn(K, N, generator=g) * sb).to(dt)
        c = torch.empty(M, N, dtype=torch.float32)
        grid = (triton.cdiv(M, 64) * triton.cdiv(N, 64),)
        G.gemm_fxp[grid](a, b, c, M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
                         c.stride(0), c.stride(1), BLOCK_SIZE_M=64, BLOCK_SIZE_N=64,
                         BLOCK_SIZE_K=64, FRAC_BITS=f, FXP_DTYPE=TL_INT[bits])
        gemms.append(dict(a=a, b=b, frac=f, bits=bits, out=c))
    torch.save(gemms, os.path.join(OUT_DIR, "gemm.pt"))
    print("gemm", len(gemms))

    # ---------------- RMSNorm ----------------
    norms = []
    for (rows, hidden, bits, f, scale, has_res) in [
        (4, 37, 32, 16, 1.0, False), (3, 64, 64, 16, 1.0, True), (5, 31, 16, 8, 8.0, False),
        (2, 100, 32, 16, 10.0, False), (3, 16, 32, 14, 4.0, True), (2, 40, 64, 16, 300.0, False),
    ]:
        x = torch.randn(rows, hidden, generator=g) * scale
        w = 1 + 0.1 * torch.randn(hidden, generator=g)
        res = torch.randn(rows, hidden, generator=g) if has_res else x
        res_in = res.clone()
        y = torch.empty_like(x)
        RN.rms_norm_fxp_kernel[(rows,)](x, w, y, res, x.stride(0), hidden, eps=1e-6,
                                        BLOCK=triton.next_power_of_2(hidden), FRAC_BITS=f,
                                        FXP_DTYPE=TL_INT[bits], HAS_RESIDUAL=has_res)
        norms.append(dict(x=x, w=w, residual=res_in if has_res else None,
                          residual_out=res.clone() if has_res else None,
                          eps=1e-6, frac=f, bits=bits, out=y))
    torch.save(norms, os.path.join(OUT_DIR, "rms_norm.pt"))
    print("rms_norm", len(norms))

    # ---------------- attention ----------------
    atts = []
    att_cases = [
        # (qlens, seqlens, H, KVH, D, page, bits, frac, causal, window, softcap, alibi, dtype)
        ([1, 1, 1], [5, 20, 37], 8, 2, 32, 16, 32, 16, True, 0, 0.0, False, torch.bfloat16),
        ([1, 1], [17, 70], 4, 1, 128, 16, 64, 16, True, 0, 0.0, False, torch.bfloat16),
        ([7, 1, 12], [7, 30, 20], 4, 2, 32, 16, 32, 14, True, 0, 0.0, False, torch.bfloat16),
        ([9, 3], [9, 40], 2, 2, 32, 4, 32, 14, True, 6, 0.0, False, torch.float32),
        ([1, 5], [33, 21], 4, 2, 64, 16, 32, 16, True, 0, 30.0, False, torch.bfloat16),
        ([6, 1], [6, 25], 4, 4, 32, 8, 32, 16, True, 0, 0.0, True, torch.float32),
        ([10], [10], 2, 1, 32, 16, 32, 14, False, 0, 0.0, False, torch.float32),
    ]
    for (qlens, seqlens, H, KVH, D, page, bits, f, causal, window, cap, alibi, dt) in att_cases:
        R = len(qlens)
        T = sum(qlens)
        max_blocks = max((s + page - 1) // page for s in seqlens)
        nblk = R * max_blocks + 3
        perm = torch.randperm(nblk, generator=g)
        block_table = perm[: R * max_blocks].view(R, max_blocks).to(torch.int32)
        q = torch.randn(T, H, D, generator=g).to(dt)
        kv = torch.randn(nblk, 2, page, KVH, D, generator=g).to(dt)
        qsl = torch.zeros(R + 1, dtype=torch.int32)
        qsl[1:] = torch.cumsum(torch.tensor(qlens), 0)
        sl = torch.tensor(seqlens, dtype=torch.int32)
        o = torch.zeros(T, H, D, dtype=torch.float32)
        slopes = (torch.rand(H, generator=g) * 0.5).float() if alibi else None
        kc, vc = kv.unbind(1)
        scale_v = AT.prepare_log2_softmax_scale(D, None)
        alibi_buf = slopes * FP.RCP_LN2 if alibi else torch.empty(0)
        grid = (R, (max(qlens) + 63) // 64, H)
        AT.unified_attention_fxp_kernel[grid](
            Q=q, K_cache=kc, V_cache=vc, softmax_scale=scale_v, batch_start_locations=qsl,
            batch_sequence_lengths=sl, block_table=block_table, output=o,
            alibi_slopes_ptr=alibi_buf, stride_query_seq=q.stride(0), stride_query_head=q.stride(1),
            stride_key_cache_block=kc.stride(0), stride_key_cache_slot=kc.stride(1),
            stride_key_cache_head=kc.stride(2), stride_value_cache_block=vc.stride(0),
            stride_value_cache_slot=vc.stride(1), stride_value_cache_head=vc.stride(2),
            stride_output_seq=o.stride(0), stride_output_head=o.stride(1),
            stride_block_table_batch=block_table.stride(0), kv_group_size=H // KVH,
            PAGE_SIZE=page, QUERY_BLOCK_SIZE=64, HEAD_DIM_PADDED=triton.next_power_of_2(D),
            KEY_BLOCK_SIZE=64, IS_CAUSAL=causal, USE_ALIBI=alibi, HEAD_DIM=D, FRAC_BITS=f,
            HEAD_DIM_CHUNK=64, FXP_DTYPE=TL_INT[bits], LOGIT_SOFTCAP=cap, WINDOW_SIZE=window,
        )
        atts.append(dict(q=q, kv_cache=kv, query_start_loc=qsl, seq_lens=sl,
                         block_table=block_table, max_query_len=max(qlens), alibi_slopes=slopes,
                         bits=bits, frac=f, causal=causal, window=window, softcap=cap, out=o))
        print("attention case done", qlens, seqlens)
    torch.save(atts, os.path.join(OUT_DIR, "attention.pt"))

    # ---------------- log-softmax ----------------
    sms = []
    for (rows, n, bits, f) in [(3, 50, 32, 16), (2, 300, 64, 16)]:
        x = torch.randn(rows, n, generator=g) * 3
        y = torch.empty_like(x)
        SM.log_softmax_fxp_kernel[(rows,)](x, y, x.stride(0), y.stride(0), n, FRAC_BITS=f,
                                           BLOCK_N=min(triton.next_power_of_2(n), 128),
                                           FXP_DTYPE=TL_INT[bits])
        sms.append(dict(x=x, bits=bits, frac=f, out=y))
    torch.save(sms, os.path.join(OUT_DIR, "log_softmax.pt"))
    print("log_softmax", len(sms))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FXPR_REFERENCE_ROOT", "../reference"))
