"""Paged unified attention launcher (reference: fixed_point_kernels/attention.py:13-15,
398-489). Same signature as the reference's ``unified_attention_fxp`` plus two
optional performance hints (``num_kv_splits``, ``max_seq_len``); results do not
depend on either.
"""

from __future__ import annotations

import ctypes
import os

import torch

from .. import _native as N
from .fixed_point import RCP_LN2, int_bits_of


def _validate_hints() -> bool:
    return os.environ.get("FXPR_VALIDATE_HINTS", "0") not in ("", "0")


def check_max_seq_len_hint(seq_lens: torch.Tensor, max_seq_len: int) -> None:
    """Raise ``ValueError`` if ``max_seq_len`` is below any entry of ``seq_lens``."""
    longest = int(seq_lens.max()) if seq_lens.numel() else 0
    if longest > int(max_seq_len):
        raise ValueError(f"unified_attention_fxp: max_seq_len={int(max_seq_len)} is below the "
                         f"longest context in seq_lens ({longest})")


def prepare_log2_softmax_scale(head_dim, softmax_scale=None):
    """attention.py:13-15."""
    scale = 1.0 / (head_dim**0.5) if softmax_scale is None else softmax_scale
    return scale * RCP_LN2


def unified_attention_fxp(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    o: torch.Tensor,
    query_start_loc: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    max_query_len: int,
    *,
    alibi_slopes: torch.Tensor | None = None,
    fxp_dtype=torch.int32,
    is_causal: bool = True,
    softmax_scale: float | None = None,
    frac_bits: int = 14,
    block_n: int = 64,
    d_chunk: int = 64,
    logits_soft_cap: float = 0.0,
    window_size: int = 0,
    num_kv_splits: int | None = None,
    max_seq_len: int | None = None,
    use_workspace: bool = True,
):
    """Run unified prefill + decode attention on a vLLM-layout paged KV cache,
    writing into ``o``. ``block_n``/``d_chunk`` are accepted for signature
    compatibility (the reference's tile sizes; they do not change results).
    ``max_seq_len`` must bound every ``seq_lens`` entry when given: keys
    beyond it are not read (the kernels cut each context at the workspace
    sized from the hint rather than overrun it). With ``FXPR_VALIDATE_HINTS=1``
    in the environment the hint is checked against ``seq_lens`` before the
    launch (a device-to-host read, so not during stream capture) and a
    violation raises ``ValueError``.
    ``use_workspace=False`` selects the scratch-free cluster path (same
    results; the chunked path is faster for decode)."""
    assert q.is_cuda and kv_cache.is_cuda, "unified_attention_fxp requires CUDA tensors"
    assert kv_cache.ndim == 5 and kv_cache.shape[1] == 2, (
        "kv_cache must be (num_blocks, 2, block_size, num_kv_heads, head_dim); "
        f"got {tuple(kv_cache.shape)}"
    )
    key_cache, value_cache = kv_cache.unbind(1)
    head_dim_query, head_dim = q.shape[-1], key_cache.shape[-1]
    assert head_dim_query == head_dim, "head_dim mismatch between q and key_cache"
    bits = int_bits_of(fxp_dtype)
    if alibi_slopes is not None:
        assert alibi_slopes.is_cuda and alibi_slopes.dtype == torch.float32, (
            "alibi_slopes must be a float32 CUDA tensor (pre-scaled by RCP_LN2)"
        )
        alibi_slopes = alibi_slopes.contiguous()
    num_requests = seq_lens.shape[0]
    if num_requests == 0 or max_query_len <= 0:
        return
    if max_seq_len and _validate_hints() and not torch.cuda.is_current_stream_capturing():
        check_max_seq_len_hint(seq_lens, max_seq_len)
    assert key_cache.stride(-1) == 1 and value_cache.stride(-1) == 1 and q.stride(-1) == 1 \
        and o.stride(-1) == 1, "head_dim must be the innermost (contiguous) dimension"
    if num_kv_splits is None:
        from ..vllm_modules.config import get_runtime_config

        num_kv_splits = get_runtime_config().num_kv_splits
    qsl = query_start_loc if query_start_loc.dtype == torch.int32 else query_start_loc.to(torch.int32)
    sl = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    qsl, sl = qsl.contiguous(), sl.contiguous()
    if bt.stride(-1) != 1:
        bt = bt.contiguous()
    p = N.AttentionParams()
    p.q, p.q_dtype, p.q_stride_tok, p.q_stride_head = q.data_ptr(), N.dcode(q), q.stride(0), q.stride(1)
    p.k_cache, p.v_cache, p.kv_dtype = key_cache.data_ptr(), value_cache.data_ptr(), N.dcode(key_cache)
    p.k_stride_blk, p.k_stride_slot, p.k_stride_head = key_cache.stride()[:3]
    p.v_stride_blk, p.v_stride_slot, p.v_stride_head = value_cache.stride()[:3]
    p.o, p.o_dtype, p.o_stride_tok, p.o_stride_head = o.data_ptr(), N.dcode(o), o.stride(0), o.stride(1)
    p.query_start_loc, p.seq_lens, p.block_table = qsl.data_ptr(), sl.data_ptr(), bt.data_ptr()
    p.bt_stride = bt.stride(0)
    p.block_table_cols = bt.shape[1]
    p.max_seq_len = int(max_seq_len) if max_seq_len else 0
    p.alibi_slopes = alibi_slopes.data_ptr() if alibi_slopes is not None else None
    p.num_requests = num_requests
    p.max_query_len = int(max_query_len)
    p.num_heads = q.shape[1]
    p.num_kv_heads = key_cache.shape[2]
    p.head_dim = head_dim
    p.page_size = key_cache.shape[1]
    p.num_blocks = key_cache.shape[0]
    p.is_causal = 1 if is_causal else 0
    p.window_size = int(window_size)
    p.scale_log2 = prepare_log2_softmax_scale(head_dim_query, softmax_scale)
    p.logits_soft_cap = logits_soft_cap * RCP_LN2 if logits_soft_cap > 0.0 else 0.0
    p.frac_bits = frac_bits
    p.int_bits = bits
    p.num_kv_splits = int(num_kv_splits)
    lib = N.load()
    if use_workspace:
        need = lib.fxpr_attention_workspace_bytes(ctypes.byref(p))
        ws = N.attention_workspace(q.device, need)
        if ws is not None:
            p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    rc = lib.fxpr_unified_attention_fxp(ctypes.byref(p), N.stream_ptr(q.device))
    N.check(rc, "unified_attention_fxp")
