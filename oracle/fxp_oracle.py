"""CPU restatement of the FxPR fixed-point reduction hot path.

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA
kernels of ``fxpr_vllm``: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may import it. The product path never calls
it and has no CPU fallback.

Every function restates the reference algorithm (Gursukh/Fixed-Point-
Reductions-For-vLLM, Triton 3.6 kernels) with torch CPU tensor ops, following
the reference's cast placement exactly. Citations are ``path:line`` inside the
reference project.

Notation: ``F2X`` = float_to_fixed (scale by 2^f, clamp to
[qmin, qmax_f], round-to-nearest-even, cast), ``X2F`` = fixed_to_float
(int -> float with RNE, times 2^-f). Integer accumulation wraps in two's
complement at the accumulator width, exactly like the Triton integer adds.

Parity pinning: the integer parts (casts, GEMM, the squared-sum of RMSNorm,
the attention score/normaliser/PV integer sums) are exact and pinned by the
golden vectors under ``tests/golden`` (outputs of the reference's own kernels
run through the Triton CPU interpreter, see ``tests/golden/make_golden.py``).
The few float primitives that the reference leaves to the GPU compiler
(``exp2``, the fast ``/`` and ``sqrt``) are injected through :class:`Prims`:
``NUMPY_PRIMS`` reproduces the Triton interpreter (used for the golden
vectors); GPU tests inject the device primitives of the CUDA library so that
the comparison with the kernels is bitwise.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

# fixed_point.py:4
RCP_LN2 = 1.4426950408889634

_INT_DTYPE = {16: torch.int16, 32: torch.int32, 64: torch.int64}
# mantissa width + 1 per float dtype (fixed_point.py:42 uses fp_mantissa_width + 1)
_MANT = {torch.float16: 11, torch.float32: 24, torch.float64: 53}


def int_dtype(int_bits: int) -> torch.dtype:
    """fixed_point.py:9-14: 16/32/64 -> signed int dtype, ValueError otherwise."""
    try:
        return _INT_DTYPE[int_bits]
    except KeyError:
        raise ValueError(f"fxp_int_bits must be 16/32/64, got {int_bits}") from None


def clamp_bounds(float_dtype: torch.dtype, int_bits: int) -> tuple[float, float]:
    """fixed_point.py:41-46: qmin_f / qmax_f as Python floats (before the
    conversion to the input dtype that Triton applies to the constants)."""
    mant = _MANT[float_dtype]
    safe_shift = 0 if int_bits <= mant else int_bits - mant
    qmax_f = float((1 << (int_bits - 1)) - (1 << safe_shift))
    qmin_f = float(-(1 << (int_bits - 1)))
    return qmin_f, qmax_f


def wrap_int(v: torch.Tensor, int_bits: int) -> torch.Tensor:
    """Two's-complement wrap of an int64 tensor to ``int_bits`` bits."""
    v = v.to(torch.int64)
    if int_bits == 64:
        return v
    m = 1 << int_bits
    h = 1 << (int_bits - 1)
    return ((v + h) % m) - h


def float_to_fixed(x: torch.Tensor, frac_bits: int, int_bits: int) -> torch.Tensor:
    """fixed_point.py:25-53.

    ``scaled = x * 2^f`` and the clamp run in x's own dtype (Triton converts
    the Python constants to x's dtype; for fp16 large constants become inf).
    NaN maps to qmin: ``tl.maximum``/``tl.minimum`` lower to maxnum/minnum on
    the GPU, which return the non-NaN operand. The final cast saturates
    (PTX float->int conversion), which only matters for fp16 inputs where the
    clamp constants overflow to inf.
    """
    if x.dtype not in _MANT:
        raise TypeError(f"x must be float16/float32/float64, got {x.dtype}")
    idt = int_dtype(int_bits)
    qmin_f, qmax_f = clamp_bounds(x.dtype, int_bits)
    # Triton materialises Python float constants as fp32 first, then casts
    # them to x's dtype (for fp64 x, qmax 2^31-1 becomes 2^31 and the final
    # conversion saturates).
    scale = torch.tensor(2.0**frac_bits, dtype=torch.float32).to(x.dtype)
    qmin = torch.tensor(qmin_f, dtype=torch.float32).to(x.dtype)
    qmax = torch.tensor(qmax_f, dtype=torch.float32).to(x.dtype)
    scaled = x * scale
    nan = torch.isnan(scaled)
    clamped = torch.minimum(torch.maximum(scaled, qmin), qmax)
    clamped = torch.where(nan, qmin.expand_as(clamped), clamped)
    r = torch.round(clamped.to(torch.float64))  # RNE, exact in float64
    lo = float(-(1 << (int_bits - 1)))
    pos_over = r >= 2.0 ** (int_bits - 1)
    neg_over = r < lo
    safe = torch.where(pos_over | neg_over, torch.zeros_like(r), r)
    out = safe.to(torch.int64)
    out[pos_over] = (1 << (int_bits - 1)) - 1
    out[neg_over] = -(1 << (int_bits - 1))
    return out.to(idt)


def fixed_to_float(q: torch.Tensor, frac_bits: int, float_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """fixed_point.py:56-69: ``q.to(float) * 2^-f`` in the float dtype."""
    q64 = q.to(torch.int64)
    if float_dtype == torch.float64:
        f = q64.to(torch.float64)
    elif float_dtype == torch.float32:
        f = q64.to(torch.float32)  # single RNE rounding int64 -> fp32
    elif float_dtype == torch.float16:
        f = q64.to(torch.float64).to(torch.float16)
    else:
        raise TypeError(f"unsupported float dtype {float_dtype}")
    inv = torch.tensor(2.0**-frac_bits, dtype=torch.float64).to(float_dtype)
    return f * inv


# --------------------------------------------------------------------------
# float primitives the reference leaves to the GPU compiler
# --------------------------------------------------------------------------


def _np_unary(fn):
    def f(x: torch.Tensor) -> torch.Tensor:
        return torch.from_numpy(np.asarray(fn(x.to(torch.float32).numpy())).astype(np.float32))

    return f


def _np_div(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    a, b = torch.broadcast_tensors(a.to(torch.float32), b.to(torch.float32))
    return torch.from_numpy(np.divide(a.numpy(), b.numpy()).astype(np.float32))


@dataclass(frozen=True)
class Prims:
    """fp32 primitives whose rounding is chosen by the compiler in the
    reference: ``tl.math.exp2`` (attention.py:237), ``/`` (attention.py:268,
    rms_norm.py:56-57), ``tl.sqrt`` (rms_norm.py:57), ``libdevice.tanh``
    (attention.py:130), ``tl.exp``/``tl.log`` (softmax.py:38, 44)."""

    exp2: Callable[[torch.Tensor], torch.Tensor]
    div: Callable[[torch.Tensor, torch.Tensor], torch.Tensor]
    sqrt: Callable[[torch.Tensor], torch.Tensor]
    tanh: Callable[[torch.Tensor], torch.Tensor]
    exp: Callable[[torch.Tensor], torch.Tensor]
    log: Callable[[torch.Tensor], torch.Tensor]
    # c + a * b of the ALiBi term (attention.py:131-135, 204-208): the Triton
    # interpreter rounds the product and the sum separately; Triton 3.6 on the
    # GPU contracts them into one fused multiply-add
    muladd: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor] = None
    # qk / cap of the softcap (attention.py:130, 203), cap a compile-time
    # constant: the interpreter divides; Triton 3.6 on the GPU multiplies by
    # the fp32 reciprocal of the constant
    div_const: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] = None


def _muladd_separate(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    return c + a * b


def mul_rcp32(a: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """a / c as the GPU build of the reference computes it for a constant c:
    a * RN(1 / c) in fp32."""
    rc = torch.tensor(1.0, dtype=torch.float32) / c.to(torch.float32)
    return a.to(torch.float32) * rc


def fma32(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """Correctly rounded fp32 fused multiply-add RN(a * b + c), computed in
    float64: the product of two fp32 values is exact in float64; the sum is
    split by TwoSum into s + e exactly, and s is rounded to fp32 with e
    deciding only when s sits exactly on an fp32 rounding midpoint."""
    a64, b64, c64 = (torch.broadcast_tensors(a.double(), b.double(), c.double()))
    x = a64 * b64
    s = x + c64
    bb = s - x
    e = (x - (s - bb)) + (c64 - bb)  # s + e == x + c exactly
    r = s.to(torch.float32)
    lo = torch.nextafter(r, torch.full_like(r, -float("inf")))
    hi = torch.nextafter(r, torch.full_like(r, float("inf")))
    # s exactly halfway between r and a neighbour: e picks the side
    up_mid = (r.double() + hi.double()) / 2 == s
    dn_mid = (r.double() + lo.double()) / 2 == s
    r = torch.where(up_mid & (e > 0), hi, r)
    r = torch.where(dn_mid & (e < 0), lo, r)
    return torch.where(torch.isfinite(s), r, (a * b + c))


NUMPY_PRIMS = Prims(
    exp2=_np_unary(np.exp2), div=_np_div, sqrt=_np_unary(np.sqrt), tanh=_np_unary(np.tanh),
    exp=_np_unary(np.exp), log=_np_unary(np.log), muladd=_muladd_separate,
)


# --------------------------------------------------------------------------
# fixed-point sum (semantics of tests/test_sum.py:13-29)
# --------------------------------------------------------------------------


def fxp_sum(x: torch.Tensor, frac_bits: int, int_bits: int = 32) -> torch.Tensor:
    """Row sums over the last dim: per-element F2X in int_b, exact int64
    sum, saturating clamp to the full int_b range, X2F to fp32
    (tests/test_sum.py:13-29: ``fixed_sum`` + ``fixed_sum_as_float``).
    bfloat16 input is widened exactly to fp32 first."""
    if x.dtype == torch.bfloat16:
        x = x.to(torch.float32)
    q = float_to_fixed(x, frac_bits, int_bits).to(torch.int64)
    acc = q.sum(dim=-1)  # int64, wraps mod 2^64 like torch's int64 sum
    info = torch.iinfo(int_dtype(int_bits))
    acc = acc.clamp(info.min, info.max)
    return fixed_to_float(acc, frac_bits, torch.float32)


# --------------------------------------------------------------------------
# fixed-point GEMM (gemm.py:7-46, 97-131, 134-196; library_ops.py:14-45)
# --------------------------------------------------------------------------


def gemm_fxp_int(a: torch.Tensor, b: torch.Tensor, frac_bits: int, int_bits: int,
                 k_chunk: int = 64) -> torch.Tensor:
    """Integer accumulator of the fixed-point GEMM, wrapped to int_b bits.

    Per product: ``fp32(a[m,k]) * fp32(b[k,n])`` (one RN fp32 multiply,
    gemm.py:42-44), F2X into int_b (gemm.py:45), integer add that wraps at
    int_b (gemm.py:45, 116-129). Integer addition is associative, so the
    sum order is free; the result is the int64 sum wrapped to int_b.
    """
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    af = a.to(torch.float32)
    bf = b.to(torch.float32)
    acc = torch.zeros((M, N), dtype=torch.int64)
    for k0 in range(0, K, k_chunk):
        k1 = min(K, k0 + k_chunk)
        prod = af[:, k0:k1, None] * bf[None, k0:k1, :]
        acc += float_to_fixed(prod, frac_bits, int_bits).to(torch.int64).sum(dim=1)
    return wrap_int(acc, int_bits)


def gemm_fxp(a: torch.Tensor, b: torch.Tensor, frac_bits: int, int_bits: int) -> torch.Tensor:
    """``fxpr::gemm_fxp``: fp32 C = X2F(integer accumulator) (gemm.py:131)."""
    return fixed_to_float(gemm_fxp_int(a, b, frac_bits, int_bits), frac_bits, torch.float32)


def linear_apply(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                 frac_bits: int, int_bits: int) -> torch.Tensor:
    """FixedPointLinearMethod.apply (quantisation_config.py:163-187): x cast to
    the weight dtype (bf16), fp32 GEMM out, ``+ bias.float()``, cast back."""
    x2d = x.reshape(-1, x.shape[-1]).to(weight.dtype)
    out = gemm_fxp(x2d, weight.t(), frac_bits, int_bits)
    out = out.view(*x.shape[:-1], out.shape[-1])
    if bias is not None:
        out = out + bias.to(torch.float32)
    return out.to(x.dtype)


# --------------------------------------------------------------------------
# RMSNorm (rms_norm.py:10-60; library_ops.py:53-126)
# --------------------------------------------------------------------------


def rms_norm_fxp(x: torch.Tensor, weight: torch.Tensor, eps: float, frac_bits: int,
                 int_bits: int, residual: torch.Tensor | None = None,
                 prims: Prims = NUMPY_PRIMS):
    """Triton kernel semantics, one row at a time (rms_norm.py:32-60).

    Returns ``y`` (x's dtype), and the updated residual (residual's dtype)
    when ``residual`` is given.
    """
    shape = x.shape
    hidden = shape[-1]
    x2 = x.reshape(-1, hidden).to(torch.float32)
    w = weight.to(torch.float32)
    new_res = None
    if residual is not None:
        r2 = residual.reshape(-1, hidden).to(torch.float32)
        x2 = x2 + r2  # rms_norm.py:43
        new_res = x2.to(residual.dtype).view(residual.shape)
    x_sq = x2 * x2  # rms_norm.py:46
    q = float_to_fixed(x_sq, frac_bits, int_bits).to(torch.int64)
    # tl.sum promotes int16 to int32 (triton/language/standard.py _pick_sum_dtype)
    sum_bits = 32 if int_bits == 16 else int_bits
    s = wrap_int(q.sum(dim=-1), sum_bits)
    sum_float = fixed_to_float(s, frac_bits, torch.float32)
    mean_sq = prims.div(sum_float, torch.tensor(float(hidden), dtype=torch.float32))
    mean_sq = torch.clamp_min(mean_sq, 0.0)  # rms_norm.py:56
    eps32 = torch.tensor(eps, dtype=torch.float64).to(torch.float32)
    rrms = prims.div(torch.ones((), dtype=torch.float32), prims.sqrt(mean_sq + eps32))
    y = (x2 * w) * rrms[:, None]  # rms_norm.py:59
    y = y.to(x.dtype).view(shape)
    if residual is not None:
        return y, new_res
    return y


def rms_norm_det_torch(x_fp32: torch.Tensor, weight: torch.Tensor, eps: float,
                       frac_bits: int, int_bits: int) -> torch.Tensor:
    """The reference's own CPU path, ``DeterministicRMSNorm._det_norm_torch``
    (vllm_modules/rms_norm.py:21-41). Differs from the Triton kernel only at
    saturation (round before clamp, clamp to 2^(b-1)-1, no int wrap) and in
    the ulp of rsqrt. Used as the timed reference CPU implementation."""
    int_dt = int_dtype(int_bits)
    scale = float(1 << frac_bits)
    qmax = (1 << (int_bits - 1)) - 1
    qmin = -(1 << (int_bits - 1))
    sq = x_fp32 * x_fp32
    scaled = (sq * scale).round().clamp_(qmin, qmax).to(int_dt)
    sum_int = scaled.sum(dim=-1, dtype=torch.int64)
    sum_fp = sum_int.to(torch.float32) / scale
    mean_sq = (sum_fp / x_fp32.shape[-1]).clamp_min_(0.0)
    rrms = torch.rsqrt(mean_sq + eps)
    return x_fp32 * weight.to(torch.float32) * rrms.unsqueeze(-1)


# --------------------------------------------------------------------------
# paged attention (attention.py:13-15, 18-279, 282-395, 398-489)
# --------------------------------------------------------------------------


def log2_softmax_scale(head_dim: int, softmax_scale: float | None) -> float:
    """attention.py:13-15 (Python double; the kernel receives it as fp32)."""
    scale = 1.0 / (head_dim**0.5) if softmax_scale is None else softmax_scale
    return scale * RCP_LN2


def unified_attention_fxp(q, kv_cache, o, query_start_loc, seq_lens, block_table,
                          max_query_len: int, *, alibi_slopes=None, int_bits: int = 32,
                          is_causal: bool = True, softmax_scale: float | None = None,
                          frac_bits: int = 14, logits_soft_cap: float = 0.0,
                          window_size: int = 0, prims: Prims = NUMPY_PRIMS,
                          query_block_size: int = 64):
    """Unified prefill+decode paged attention (attention.py:398-489 launcher,
    282-395 program, 18-279 body), one (request, q-block, head) program at a
    time. Writes into ``o`` and returns it.

    ``alibi_slopes`` are pre-scaled by RCP_LN2 (attention.py:433-435).
    ``int_bits`` selects the fixed-point accumulator (the reference's
    ``fxp_dtype``); 16 is rejected: the reference's int16 attention fails to
    compile (the loop-carried int16 denominator is promoted to int32 by
    tl.sum, attention.py:150, 243).
    """
    if int_bits == 16:
        raise ValueError("int16 accumulators are not supported by the attention kernel")
    assert kv_cache.ndim == 5 and kv_cache.shape[1] == 2
    key_cache = kv_cache[:, 0]
    value_cache = kv_cache[:, 1]
    D = q.shape[-1]
    assert key_cache.shape[-1] == D
    scale32 = torch.tensor(log2_softmax_scale(D, softmax_scale), dtype=torch.float64).to(torch.float32)
    num_requests = seq_lens.shape[0]
    H = q.shape[1]
    KVH = key_cache.shape[2]
    group = H // KVH
    page = key_cache.shape[1]
    QB = query_block_size
    max_q_blocks = (max_query_len + QB - 1) // QB
    if num_requests == 0 or max_q_blocks == 0:
        return o
    cap_log2 = torch.tensor(logits_soft_cap * RCP_LN2, dtype=torch.float64).to(torch.float32)
    neg_inf = torch.tensor(float("-inf"), dtype=torch.float32)
    tiny = torch.tensor(1.0e-6, dtype=torch.float32)
    qsl = query_start_loc.to(torch.int64).tolist()
    sl = seq_lens.to(torch.int64).tolist()
    for r in range(num_requests):
        seq_len = sl[r]
        q_start, q_end = qsl[r], qsl[r + 1]
        qlen = q_end - q_start
        ctx = seq_len - qlen
        for b in range(max_q_blocks):
            qb0 = QB * b
            if qb0 >= qlen:
                continue
            qoffs = torch.arange(qb0, min(qb0 + QB, qlen))
            pos = ctx + qoffs
            key_end = min(seq_len, ctx + (b + 1) * QB) if is_causal else seq_len
            keys = torch.arange(max(key_end, 0))
            blocks = block_table[r, keys // page].to(torch.int64)
            slots = keys % page
            for h in range(H):
                kvh = h // group
                kk = key_cache[blocks, slots, kvh].to(torch.float32)  # [J, D]
                vv = value_cache[blocks, slots, kvh].to(torch.float16).to(torch.float32)
                qq = q[q_start + qoffs, h].to(torch.float32)  # [I, D]
                # score: sum_d F2X(q*k) in int_b (gemm.py:7-46 via attention.py:107-117)
                prod = qq[:, None, :] * kk[None, :, :]
                s_int = wrap_int(float_to_fixed(prod, frac_bits, int_bits).to(torch.int64).sum(-1), int_bits)
                qk = fixed_to_float(s_int, frac_bits, torch.float32) * scale32
                if logits_soft_cap > 0.0:
                    qk = cap_log2 * prims.tanh((prims.div_const or prims.div)(qk, cap_log2))
                if alibi_slopes is not None:
                    slope = alibi_slopes[h].to(torch.float32)
                    diff = keys[None, :].to(torch.float32) - pos[:, None].to(torch.float32)
                    qk = (prims.muladd or _muladd_separate)(slope, diff, qk)
                mask = torch.ones((len(qoffs), len(keys)), dtype=torch.bool)
                if is_causal:
                    mask &= pos[:, None] >= keys[None, :]
                if window_size > 0:
                    mask &= keys[None, :] > (pos[:, None] - window_size)
                qk = torch.where(mask, qk, neg_inf)
                if len(keys):
                    row_max = qk.max(dim=1).values  # attention.py:148
                else:
                    row_max = torch.full((len(qoffs),), float("-inf"))
                p = prims.exp2(qk - row_max[:, None])  # attention.py:237
                den = wrap_int(float_to_fixed(p, frac_bits, int_bits).to(torch.int64).sum(-1), int_bits)
                pv = p[:, :, None] * vv[None, :, :]  # attention.py:253 via gemm.py:49-71
                acc = wrap_int(float_to_fixed(pv, frac_bits, int_bits).to(torch.int64).sum(1), int_bits)
                den_f = fixed_to_float(den, frac_bits, torch.float32)
                acc_f = fixed_to_float(acc, frac_bits, torch.float32)
                den_safe = torch.maximum(den_f, tiny)
                out = prims.div(acc_f, den_safe[:, None])  # attention.py:267-268
                o[q_start + qoffs, h] = out.to(o.dtype)
    return o


# --------------------------------------------------------------------------
# log-softmax for sampler logprobs (softmax.py:8-52, 55-97)
# --------------------------------------------------------------------------


def log_softmax_fxp(x: torch.Tensor, int_bits: int, frac_bits: int = 16,
                    prims: Prims = NUMPY_PRIMS) -> torch.Tensor:
    """Row-wise log-softmax over the last dim with a fixed-point exp-sum.
    Logits are rounded to fp16 before the max and the exp (softmax.py:27-28,
    36-37, 50); the integer exp-sum wraps at int_b (softmax.py:41-42)."""
    orig = x.dtype
    x16 = x.to(torch.float32).to(torch.float16).to(torch.float32)
    row_max = x16.max(dim=-1, keepdim=True).values
    e = prims.exp(x16 - row_max)
    s = float_to_fixed(e, frac_bits, int_bits).to(torch.int64).sum(-1, keepdim=True)
    s = wrap_int(s, int_bits)
    ls = prims.log(fixed_to_float(s, frac_bits, torch.float32))
    return ((x16 - row_max) - ls).to(orig)


__all__ = [
    "RCP_LN2", "Prims", "NUMPY_PRIMS", "int_dtype", "clamp_bounds", "wrap_int",
    "float_to_fixed", "fixed_to_float", "fxp_sum", "gemm_fxp_int", "gemm_fxp",
    "linear_apply", "rms_norm_fxp", "rms_norm_det_torch", "log2_softmax_scale",
    "unified_attention_fxp", "log_softmax_fxp",
]
