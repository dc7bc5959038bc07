"""ctypes binding of the C ABI in ``include/fxpr_b200.h``.

The CUDA library ``_lib/libfxpr_b200.so`` is built in-tree (``build.py``).
There is no fallback: if the library is missing or a tensor is not on a CUDA
device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

# FXPR_B200_LIB: another build of the same library (e.g. with different tile
# constants); default is the in-tree build
_LIB_PATH = os.environ.get("FXPR_B200_LIB") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), "_lib", "libfxpr_b200.so")

FXPR_OK = 0
FXPR_ERR_INVALID = -1
FXPR_ERR_UNSUPPORTED = -2
FXPR_ERR_CUDA = -3

F16, BF16, F32, F64, I16, I32, I64 = 0, 1, 2, 3, 10, 11, 12
DTYPE_CODE = {
    torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.float64: F64,
    torch.int16: I16, torch.int32: I32, torch.int64: I64,
}

# every symbol the header declares
EXPORTED = (
    "fxpr_abi_version", "fxpr_last_error", "fxpr_float_to_fixed", "fxpr_fixed_to_float",
    "fxpr_fxp_sum", "fxpr_gemm_workspace_bytes", "fxpr_gemm_fxp", "fxpr_fixed_to_float_bias",
    "fxpr_rms_norm_fxp", "fxpr_unified_attention_fxp", "fxpr_log_softmax_fxp", "fxpr_probe_prims",
    "fxpr_gemm_fxp_noalloc", "fxpr_attention_workspace_bytes", "fxpr_fixed_to_float_add_rms_norm",
)

_i = ctypes.c_int
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_f = ctypes.c_float


class AttentionParams(ctypes.Structure):
    """Mirror of ``fxpr_attention_params``."""

    _fields_ = [
        ("q", _p), ("q_dtype", _i), ("q_stride_tok", _i64), ("q_stride_head", _i64),
        ("k_cache", _p), ("v_cache", _p), ("kv_dtype", _i),
        ("k_stride_blk", _i64), ("k_stride_slot", _i64), ("k_stride_head", _i64),
        ("v_stride_blk", _i64), ("v_stride_slot", _i64), ("v_stride_head", _i64),
        ("o", _p), ("o_dtype", _i), ("o_stride_tok", _i64), ("o_stride_head", _i64),
        ("query_start_loc", _p), ("seq_lens", _p), ("block_table", _p), ("bt_stride", _i64),
        ("block_table_cols", ctypes.c_int32), ("max_seq_len", ctypes.c_int32),
        ("alibi_slopes", _p),
        ("num_requests", ctypes.c_int32), ("max_query_len", ctypes.c_int32),
        ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("page_size", ctypes.c_int32),
        ("is_causal", ctypes.c_int32), ("window_size", ctypes.c_int32),
        ("scale_log2", _f), ("logits_soft_cap", _f),
        ("frac_bits", ctypes.c_int32), ("int_bits", ctypes.c_int32),
        ("num_kv_splits", ctypes.c_int32),
        ("workspace", _p), ("workspace_bytes", _i64),
        ("num_blocks", _i64),
    ]


_SIGS = {
    "fxpr_abi_version": (_i, []),
    "fxpr_last_error": (ctypes.c_char_p, []),
    "fxpr_float_to_fixed": (_i, [_p, _i, _p, _i, _i64, _i, _p]),
    "fxpr_fixed_to_float": (_i, [_p, _i, _p, _i, _i64, _i, _p]),
    "fxpr_fxp_sum": (_i, [_p, _i, _i64, _i64, _i64, _p, _i, _i, _p]),
    "fxpr_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64, _i]),
    "fxpr_gemm_fxp": (_i, [_p, _i, _i64, _i64, _p, _i, _i64, _i64, _p, _i, _i64, _i64,
                           _i64, _i64, _i64, _i, _i, _p, _i64, _p]),
    "fxpr_gemm_fxp_noalloc": (_i, [_p, _i, _i64, _i64, _p, _i, _i64, _i64, _p, _i, _i64, _i64,
                                   _i64, _i64, _i64, _i, _i, _p]),
    "fxpr_fixed_to_float_bias": (_i, [_p, _i, _i64, _i64, _i64, _p, _i, _p, _i, _i64, _i, _p]),
    "fxpr_rms_norm_fxp": (_i, [_p, _i, _i64, _p, _i, _p, _i, _i64, _p, _i, _i64, _i64, _i64,
                               _f, _i, _i, _p]),
    "fxpr_fixed_to_float_add_rms_norm": (_i, [_p, _i, _i64, _p, _i, _p, _i, _i64, _p, _i, _p, _i64,
                                              _i64, _i64, _f, _i, _p]),
    "fxpr_unified_attention_fxp": (_i, [ctypes.POINTER(AttentionParams), _p]),
    "fxpr_attention_workspace_bytes": (_i64, [ctypes.POINTER(AttentionParams)]),
    "fxpr_log_softmax_fxp": (_i, [_p, _i64, _p, _i64, _i64, _i64, _i, _i, _p]),
    "fxpr_probe_prims": (_i, [_i, _p, _p, _p, _i64, _p]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"fxpr_vllm: CUDA library not built ({_LIB_PATH}); run "
                    "`python fixed-point-reductions-for-vllm_b200/build.py`"
                )
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc == FXPR_OK:
        return
    msg = load().fxpr_last_error().decode(errors="replace")
    if rc == FXPR_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    if rc == FXPR_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("fxpr_vllm kernels require CUDA tensors (no CPU fallback)")
        dev = t.device if dev is None else dev
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dcode(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# --------------------------------------------------------------------------
# Kernel scratch: one buffer per (kind, device, stream). The GEMM's split-K
# scratch is left zero-filled by every call; the attention scratch carries no
# state between calls.
#
# A buffer is never freed once handed out: a CUDA graph captured on the same
# stream records its address, and replays keep writing there. When a larger
# call needs more room, the new buffer replaces the old one for later calls,
# and the old one moves to ``_retired`` (kept alive for the life of the
# process). Growth is geometric, so few buffers are ever retired.
# --------------------------------------------------------------------------
_ws: dict[tuple[str, int, int], torch.Tensor] = {}
_retired: list[torch.Tensor] = []


def _workspace(kind: str, device: torch.device, nbytes: int) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    key = (kind, device.index if device.index is not None else torch.cuda.current_device(),
           stream_ptr(device))
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if buf is not None:
            size = max(size, 2 * buf.numel())
            _retired.append(buf)
        buf = torch.zeros(size, dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf


def gemm_workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    return _workspace("gemm", device, nbytes)


def attention_workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Scratch of the chunked attention path (no state between calls)."""
    return _workspace("attn", device, nbytes)
