"""End to end through vLLM: greedy token streams of a random-init
Llama-architecture model under quantization="fixed_point_det" and
attention_backend="CUSTOM" are identical across batch sizes, and the
fixed-point GEMM, RMSNorm and attention kernels are the ones that run."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fixed-point-reductions-for-vllm_b200")

SCRIPT = r"""
import json, os, sys
sys.path.insert(0, {pkg!r})
import torch
from fxpr_vllm import e2e
d = e2e.make_llama_dir({mdir!r}, "tiny", seed=0)
llm = e2e.make_llm(d, max_num_seqs=16, gpu_mem=0.25, max_model_len=512, enforce_eager=True)
ps = e2e.prompts(8, 40, 1024, seed=1)
with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
    full = e2e.generate(llm, ps, 24)
names = sorted({{e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}})
one = e2e.generate(llm, ps, 24, batch=1)
three = e2e.generate(llm, ps, 24, batch=3)
json.dump({{"full": full, "one": one, "three": three, "kernels": names}}, open({out!r}, "w"))
"""


def test_greedy_streams_identical_and_fixed_point_kernels_used(tmp_path):
    out = tmp_path / "streams.json"
    code = SCRIPT.format(pkg=PKG, mdir=str(tmp_path / "tiny"), out=str(out))
    env = dict(os.environ, PYTHONPATH=PKG, VLLM_ENABLE_V1_MULTIPROCESSING="0",
               VLLM_HOST_IP="127.0.0.1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    a = json.load(open(out))
    assert a["full"] == a["one"] == a["three"]
    assert all(len(s) == 24 for s in a["full"])
    ks = " ".join(a["kernels"])
    # the fixed-point GEMM, RMSNorm, prefill attention (chunked kernels) and
    # decode attention (persistent decode kernels)
    for k in ("gemm_kc_kernel", "rms_norm", "chunk_scores", "chunk_pv_kernel", "dq_scores_kernel",
              "dq_pv_kernel"):
        assert k in ks, (k, a["kernels"])
    # no float GEMM left: the LM head runs the fixed-point GEMM too
    assert not any("nvjet" in k or "cublas" in k.lower() for k in a["kernels"]), a["kernels"]
