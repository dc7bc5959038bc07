"""Build recipe of the compiled reference checker ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY. Compiles the reference plugin's own Triton kernels
(Gursukh/Fixed-Point-Reductions-For-vLLM, read in place from the reference
checkout, never copied) ahead of time for sm_100 with the Triton that is
installed here, into cubins plus a small JSON of launch metadata under
``oracle/_ref/``. That directory is git-ignored and travels to the GPU box
with the rest of the working tree; ``oracle/ref_triton.py`` loads and
launches the cubins there, so the GPU tests can compare the CUDA kernels with
the reference kernels *as Triton lowers them on B200* (its exp2, fast divide
and square root, and its floating-point contraction choices), and so the
benchmark can time them as the device baseline.

Kernels and the reference launch each specialisation mirrors:

* ``unified_attention_fxp_kernel`` (fixed_point_kernels/attention.py:282-395),
  launched as attention.py:440-489 (num_warps 4 for head_dim <= 64 else 8,
  num_stages 1, query block 64, key block 64, d_chunk 64);
* ``rms_norm_fxp_kernel`` (fixed_point_kernels/rms_norm.py:10-60), launched as
  library_ops.py:53-126 (default num_warps / num_stages, BLOCK = next power
  of two of hidden);
* ``gemm_fxp`` (fixed_point_kernels/gemm.py:134-196), launched as
  library_ops.py:14-45 (64 x 64 x 64 blocks);
* ``log_softmax_fxp_kernel`` (fixed_point_kernels/softmax.py:8-52), launched
  as softmax.py:55-97 (BLOCK_N = min(next power of two of N, 1024)).

The softcap specialisation reads the module global ``RCP_LN2`` inside the jit
function (attention.py:129, 202), which Triton 3.6 only accepts with
``TRITON_ALLOW_NON_CONSTEXPR_GLOBALS=1``; the build sets it (the reference's
softcap path does not compile on a stock Triton 3.6 without it).

Integer arguments are compiled as i32 and pointers without alignment hints
(the JIT would add divisibility hints; they change address arithmetic, not
the floating-point operations).

    python oracle/build_ref.py [REFERENCE_ROOT]   # default: $FXPR_REFERENCE_ROOT or DEFAULT_REF
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
DEFAULT_REF = os.environ.get("FXPR_REFERENCE_ROOT", "/root/reference")
RCP_LN2 = 1.4426950408889634


def _attention_specs(tl):
    specs = []
    base = dict(PAGE_SIZE=16, QUERY_BLOCK_SIZE=64, KEY_BLOCK_SIZE=64, IS_CAUSAL=True,
                USE_ALIBI=False, FRAC_BITS=16, HEAD_DIM_CHUNK=64, LOGIT_SOFTCAP=0.0,
                WINDOW_SIZE=0)
    for D, G, bits in [(128, 4, 32), (128, 4, 64), (64, 4, 32)]:
        specs.append((f"attn_d{D}_g{G}_i{bits}", dict(base, kv_group_size=G, HEAD_DIM=D,
                                                      HEAD_DIM_PADDED=D, FXP_DTYPE=bits)))
    specs.append(("attn_d128_g4_i32_alibi", dict(base, kv_group_size=4, HEAD_DIM=128,
                                                 HEAD_DIM_PADDED=128, FXP_DTYPE=32, USE_ALIBI=True)))
    specs.append(("attn_d128_g4_i32_softcap30", dict(base, kv_group_size=4, HEAD_DIM=128,
                                                     HEAD_DIM_PADDED=128, FXP_DTYPE=32,
                                                     LOGIT_SOFTCAP=30.0)))
    specs.append(("attn_d128_g4_i32_window100", dict(base, kv_group_size=4, HEAD_DIM=128,
                                                     HEAD_DIM_PADDED=128, FXP_DTYPE=32,
                                                     WINDOW_SIZE=100)))
    return specs


def build(ref_root: str = DEFAULT_REF, verbose: bool = True) -> list[str]:
    """Compile every specialisation into OUT; returns the names built.
    Skips (returns []) when the reference checkout is absent."""
    if not os.path.isdir(os.path.join(ref_root, "fxpr_vllm")):
        if verbose:
            print(f"build_ref: no reference checkout at {ref_root}; skipped")
        return []
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    os.environ.setdefault("TRITON_ALLOW_NON_CONSTEXPR_GLOBALS", "1")
    import triton
    import triton.language as tl
    from triton.backends.compiler import GPUTarget
    from triton.compiler import ASTSource

    import fxpr_vllm.fixed_point_kernels.attention as ra
    import fxpr_vllm.fixed_point_kernels.gemm as rg
    import fxpr_vllm.fixed_point_kernels.rms_norm as rr
    import fxpr_vllm.fixed_point_kernels.softmax as rs

    dt = {16: tl.int16, 32: tl.int32, 64: tl.int64}
    os.makedirs(OUT, exist_ok=True)
    target = GPUTarget("cuda", 100, 32)
    built = []

    def compile_one(name, jit_fn, ptr_types, scalar_types, consts, num_warps, num_stages):
        import inspect

        params = list(inspect.signature(jit_fn.fn).parameters)
        sig = {}
        for p in params:
            if p in consts:
                sig[p] = "constexpr"
            elif p in ptr_types:
                sig[p] = ptr_types[p]
            else:
                sig[p] = scalar_types.get(p, "i32")
        cvals = {}
        for k, v in consts.items():
            if k == "FXP_DTYPE":
                v = dt[v]
            cvals[(params.index(k),)] = v
        src_file = inspect.getsourcefile(jit_fn.fn)
        with open(src_file, "rb") as f:
            digest = hashlib.sha256(f.read()).hexdigest()[:16]
        meta_path = os.path.join(OUT, name + ".json")
        key = {"triton": triton.__version__, "source": digest, "consts": repr(sorted(consts.items())),
               "warps": num_warps, "stages": num_stages, "sig": sig}
        if os.path.exists(meta_path) and os.path.exists(os.path.join(OUT, name + ".cubin")):
            with open(meta_path) as f:
                if json.load(f).get("key") == key:
                    built.append(name)
                    return
        k = triton.compile(ASTSource(fn=jit_fn, signature=sig, constexprs=cvals), target=target,
                           options={"num_warps": num_warps, "num_stages": num_stages})
        with open(os.path.join(OUT, name + ".cubin"), "wb") as f:
            f.write(k.asm["cubin"])
        args = [(p, sig[p]) for p in params if sig[p] != "constexpr"]
        meta = {"kernel": k.metadata.name, "num_warps": k.metadata.num_warps,
                "shared": k.metadata.shared, "args": args, "key": key,
                "global_scratch_size": getattr(k.metadata, "global_scratch_size", 0),
                "profile_scratch_size": getattr(k.metadata, "profile_scratch_size", 0)}
        with open(meta_path, "w") as f:
            json.dump(meta, f, indent=1)
        built.append(name)
        if verbose:
            print(f"build_ref: {name}")

    # attention (attention.py:440-489)
    aptr = {"Q": "*bf16", "K_cache": "*bf16", "V_cache": "*bf16", "batch_start_locations": "*i32",
            "batch_sequence_lengths": "*i32", "block_table": "*i32", "output": "*fp32",
            "alibi_slopes_ptr": "*fp32"}
    for name, consts in _attention_specs(tl):
        compile_one(name, ra.unified_attention_fxp_kernel, aptr, {"softmax_scale": "fp32"}, consts,
                    4 if consts["HEAD_DIM"] <= 64 else 8, 1)
    # RMSNorm (library_ops.py:53-126): the glue passes fp32 x / residual / weight
    rptr = {"X_ptr": "*fp32", "W_ptr": "*fp32", "Y_ptr": "*fp32", "Residual_ptr": "*fp32"}
    for bits in (16, 32, 64):
        for res in (False, True):
            for hidden, eps in ((4096, 1e-6), (4096, 1e-5)):
                compile_one(f"rms_h{hidden}_i{bits}_r{int(res)}_eps{eps:g}", rr.rms_norm_fxp_kernel, rptr, {},
                            dict(eps=eps, BLOCK=triton.next_power_of_2(hidden), FRAC_BITS=16 if bits > 16 else 8,
                                 FXP_DTYPE=bits, HAS_RESIDUAL=res), 4, 3)
    # GEMM (library_ops.py:14-45)
    gptr = {"a_ptr": "*bf16", "b_ptr": "*bf16", "c_ptr": "*fp32"}
    for bits in (32, 64):
        compile_one(f"gemm_bf16_i{bits}", rg.gemm_fxp, gptr, {},
                    dict(BLOCK_SIZE_M=64, BLOCK_SIZE_N=64, BLOCK_SIZE_K=64, FRAC_BITS=16, FXP_DTYPE=bits),
                    4, 3)
    # log-softmax (softmax.py:55-97)
    sptr = {"X_ptr": "*fp32", "Y_ptr": "*fp32"}
    for bits in (32, 64):
        compile_one(f"log_softmax_n1024_i{bits}", rs.log_softmax_fxp_kernel, sptr, {},
                    dict(FRAC_BITS=16, BLOCK_N=1024, FXP_DTYPE=bits), 4, 3)
    return built


if __name__ == "__main__":
    names = build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF)
    print(f"build_ref: {len(names)} kernels in {OUT}")
