"""End to end through vLLM: greedy token streams of a random-init
Llama-architecture model under quantization="fixed_point_det" and
attention_backend="CUSTOM" are identical across batch sizes and KV-split
counts (the fixed-point kernels make every reduction order-free)."""

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
from fxpr_vllm import e2e
d = e2e.make_llama_dir({mdir!r}, "tiny", seed=0)
llm = e2e.make_llm(d, max_num_seqs=16, gpu_mem=0.25, max_model_len=512)
ps = e2e.prompts(8, 40, 1024, seed=1)
full = e2e.generate(llm, ps, 24)
one = e2e.generate(llm, ps, 24, batch=1)
three = e2e.generate(llm, ps, 24, batch=3)
json.dump({{"full": full, "one": one, "three": three}}, open({out!r}, "w"))
"""


def _run(tmp_path, splits):
    out = tmp_path / f"streams_{splits}.json"
    code = SCRIPT.format(pkg=PKG, mdir=str(tmp_path / "tiny"), out=str(out))
    env = dict(os.environ, VLLM_FXP_NUM_KV_SPLITS=str(splits), PYTHONPATH=PKG)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    import json

    return json.load(open(out))


def test_greedy_streams_identical_across_batch_and_splits(tmp_path):
    a = _run(tmp_path, 8)
    assert a["full"] == a["one"] == a["three"]
    assert all(len(s) == 24 for s in a["full"])
    b = _run(tmp_path, 1)
    assert b["full"] == a["full"]
