"""Launcher of the compiled reference kernels in ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY (see ``oracle/build_ref.py``): the GPU tests use it
to run the reference plugin's own Triton kernels, compiled ahead of time for
sm_100, on the same device as the CUDA kernels and compare bit for bit; the
benchmark's device-baseline leg times them. Nothing in the product imports it.

The cubins are loaded with the CUDA driver API through ctypes into the
current (torch) context. Arguments follow Triton 3.6's kernel convention:
every non-constexpr parameter in declaration order, then the global and the
profile scratch pointers (both unused by these kernels: null).
"""

from __future__ import annotations

import ctypes
import json
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_cuda = None
_modules: dict[tuple[str, int], tuple[ctypes.c_void_p, ctypes.c_void_p, dict]] = {}


def available(name: str) -> bool:
    return os.path.exists(os.path.join(REF_DIR, name + ".cubin"))


def _driver():
    global _cuda
    if _cuda is None:
        _cuda = ctypes.CDLL("libcuda.so.1")
    return _cuda


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = ctypes.c_char_p()
        _driver().cuGetErrorString(rc, ctypes.byref(msg))
        raise RuntimeError(f"{what}: CUDA driver error {rc} ({msg.value.decode() if msg.value else '?'})")


def _load(name: str):
    dev = torch.cuda.current_device()
    key = (name, dev)
    if key in _modules:
        return _modules[key]
    torch.cuda.init()
    torch.empty(1, device="cuda")  # make the primary context current on this thread
    with open(os.path.join(REF_DIR, name + ".json")) as f:
        meta = json.load(f)
    with open(os.path.join(REF_DIR, name + ".cubin"), "rb") as f:
        image = f.read()
    cu = _driver()
    mod = ctypes.c_void_p()
    _check(cu.cuModuleLoadData(ctypes.byref(mod), ctypes.c_char_p(image)), f"cuModuleLoadData({name})")
    fn = ctypes.c_void_p()
    _check(cu.cuModuleGetFunction(ctypes.byref(fn), mod, meta["kernel"].encode()),
           f"cuModuleGetFunction({name})")
    if meta["shared"] > 48 * 1024:
        # CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8
        _check(cu.cuFuncSetAttribute(fn, 8, ctypes.c_int(meta["shared"])), "cuFuncSetAttribute")
    _modules[key] = (mod, fn, meta)
    return _modules[key]


def _arg(ty: str, v):
    if ty.startswith("*"):
        return ctypes.c_void_p(0 if v is None else (v.data_ptr() if torch.is_tensor(v) else int(v)))
    if ty == "fp32":
        return ctypes.c_float(float(v))
    if ty == "i64":
        return ctypes.c_int64(int(v))
    return ctypes.c_int32(int(v))


def launch(name: str, grid: tuple[int, int, int], **kwargs) -> None:
    """Launch reference kernel ``name`` on the current stream; keyword
    arguments name the kernel's non-constexpr parameters (tensors for
    pointers, None for a null pointer)."""
    _, fn, meta = _load(name)
    vals = [_arg(ty, kwargs[p]) for p, ty in meta["args"]]
    vals += [ctypes.c_void_p(0), ctypes.c_void_p(0)]  # global / profile scratch
    ptrs = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
    stream = torch.cuda.current_stream().cuda_stream
    gx, gy, gz = (tuple(grid) + (1, 1))[:3]
    _check(_driver().cuLaunchKernel(fn, gx, gy, gz, 32 * meta["num_warps"], 1, 1, meta["shared"],
                                    ctypes.c_void_p(stream), ptrs, None), f"cuLaunchKernel({name})")


# --------------------------------------------------------------------------
# the reference launchers, restated over `launch` (same grids and arguments)
# --------------------------------------------------------------------------


def attention(name: str, q, kv_cache, o, query_start_loc, seq_lens, block_table, max_query_len,
              softmax_scale_log2: float, alibi_slopes=None) -> None:
    """fixed_point_kernels/attention.py:398-489 with the compiled
    specialisation ``name`` (o must be fp32; alibi slopes pre-scaled by 1/ln2)."""
    key_cache, value_cache = kv_cache.unbind(1)
    num_requests = seq_lens.shape[0]
    max_q_blocks = (max_query_len + 63) // 64
    grid = (num_requests, max_q_blocks, q.shape[1])
    launch(name, grid, Q=q, K_cache=key_cache, V_cache=value_cache, softmax_scale=softmax_scale_log2,
           batch_start_locations=query_start_loc, batch_sequence_lengths=seq_lens,
           block_table=block_table, output=o, alibi_slopes_ptr=alibi_slopes,
           stride_query_seq=q.stride(0), stride_query_head=q.stride(1),
           stride_key_cache_block=key_cache.stride(0), stride_key_cache_slot=key_cache.stride(1),
           stride_key_cache_head=key_cache.stride(2), stride_value_cache_block=value_cache.stride(0),
           stride_value_cache_slot=value_cache.stride(1), stride_value_cache_head=value_cache.stride(2),
           stride_output_seq=o.stride(0), stride_output_head=o.stride(1),
           stride_block_table_batch=block_table.stride(0))


def rms_norm(name: str, x32, w32, y32, residual32=None) -> None:
    """library_ops.py:53-126 (fp32 rows; residual updated in place)."""
    rows, hidden = x32.shape
    launch(name, (rows, 1, 1), X_ptr=x32, W_ptr=w32, Y_ptr=y32, Residual_ptr=residual32,
           stride_x=x32.stride(0), hidden_size=hidden)


def gemm(name: str, a, b, c) -> None:
    """library_ops.py:14-45 (64 x 64 blocks, fp32 c)."""
    M, K = a.shape
    N = b.shape[1]
    grid = (((M + 63) // 64) * ((N + 63) // 64), 1, 1)
    launch(name, grid, a_ptr=a, b_ptr=b, c_ptr=c, M=M, N=N, K=K, stride_am=a.stride(0),
           stride_ak=a.stride(1), stride_bk=b.stride(0), stride_bn=b.stride(1),
           stride_cm=c.stride(0), stride_cn=c.stride(1))


def log_softmax(name: str, x32, y32) -> None:
    """softmax.py:55-97 (fp32 rows)."""
    rows, n = x32.shape
    launch(name, (rows, 1, 1), X_ptr=x32, Y_ptr=y32, stride_xm=x32.stride(0), stride_ym=y32.stride(0), N=n)
