"""End-to-end deterministic decode through vLLM with the fixed-point plugin.

Builds a Llama-architecture checkpoint with seeded N(0, 0.02) weights on
local disk (no network: no tokenizer, token-id prompts), then runs greedy
decode with ``quantization="fixed_point_det"`` and
``attention_backend="CUSTOM"``. Used by the GPU end-to-end test and as the
decode tokens/s benchmark (the ~1B and Llama-3-8B architecture workloads):

    python -m fxpr_vllm.e2e --preset llama1b --prompts 32 --prompt-len 512 --gen 256 --tp 1
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

PRESETS = {
    # ~1B Llama architecture
    "llama1b": dict(hidden_size=2048, num_hidden_layers=16, num_attention_heads=32,
                    num_key_value_heads=8, head_dim=64, intermediate_size=8192,
                    rms_norm_eps=1e-5, rope_theta=500000.0, vocab_size=128256),
    # Llama-3-8B architecture
    "llama8b": dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                    num_key_value_heads=8, head_dim=128, intermediate_size=14336,
                    rms_norm_eps=1e-5, rope_theta=500000.0, vocab_size=128256),
    # tiny model for tests
    "tiny": dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=8,
                 num_key_value_heads=2, head_dim=64, intermediate_size=512,
                 rms_norm_eps=1e-5, rope_theta=500000.0, vocab_size=1024),
}


def make_llama_dir(path: str, preset: str = "tiny", seed: int = 0) -> str:
    """Write config.json + model.safetensors (bf16, weights N(0, 0.02), norms 1)."""
    import torch
    from safetensors.torch import save_file

    cfg = dict(PRESETS[preset])
    os.makedirs(path, exist_ok=True)
    marker = os.path.join(path, "config.json")
    if os.path.exists(marker) and os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    conf = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "torch_dtype": "bfloat16",
        "hidden_act": "silu", "max_position_embeddings": 8192, "tie_word_embeddings": False,
        "bos_token_id": 1, "eos_token_id": 2, "attention_bias": False, "mlp_bias": False,
        **cfg,
    }
    # drawn on the GPU when there is one (seconds for 8B parameters instead of
    # minutes on the host); the same seed gives the same weights on every run
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    g = torch.Generator(device=dev).manual_seed(seed)
    H, L, I, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["intermediate_size"], cfg["vocab_size"]
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16).cpu()

    sd = {"model.embed_tokens.weight": rnd(V, H), "lm_head.weight": rnd(V, H),
          "model.norm.weight": torch.ones(H, dtype=torch.bfloat16)}
    for i in range(L):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = rnd(nh * hd, H)
        sd[p + "self_attn.k_proj.weight"] = rnd(nkv * hd, H)
        sd[p + "self_attn.v_proj.weight"] = rnd(nkv * hd, H)
        sd[p + "self_attn.o_proj.weight"] = rnd(H, nh * hd)
        sd[p + "mlp.gate_proj.weight"] = rnd(I, H)
        sd[p + "mlp.up_proj.weight"] = rnd(I, H)
        sd[p + "mlp.down_proj.weight"] = rnd(H, I)
        sd[p + "input_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
    save_file(sd, os.path.join(path, "model.safetensors"))
    with open(marker, "w") as f:
        json.dump(conf, f)
    return path


def prompts(n: int, length: int, vocab: int, seed: int = 0) -> list[list[int]]:
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, vocab, (n, length), generator=g).tolist()


def make_llm(model_dir: str, tp: int = 1, max_num_seqs: int = 256, gpu_mem: float = 0.5,
             enforce_eager: bool = False, max_model_len: int = 4096):
    pkg_root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pp = os.environ.get("PYTHONPATH", "")
    if pkg_root not in pp.split(os.pathsep):  # workers find the plugin entry point here
        os.environ["PYTHONPATH"] = pkg_root + (os.pathsep + pp if pp else "")
    if pkg_root not in sys.path:
        sys.path.insert(0, pkg_root)
    # rendezvous on loopback: the host name of the box may not resolve
    os.environ.setdefault("VLLM_HOST_IP", "127.0.0.1")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    # greedy decoding needs no FlashInfer top-k/top-p sampler, whose first use
    # JIT-compiles a module (minutes on a fresh machine)
    os.environ.setdefault("VLLM_USE_FLASHINFER_SAMPLER", "0")
    from fxpr_vllm.register import register

    register()
    from vllm import LLM

    return LLM(model=model_dir, quantization="fixed_point_det", attention_backend="CUSTOM",
               skip_tokenizer_init=True, tensor_parallel_size=tp, dtype="bfloat16",
               max_num_seqs=max_num_seqs, gpu_memory_utilization=gpu_mem,
               enforce_eager=enforce_eager, max_model_len=max_model_len, seed=0,
               enable_prefix_caching=False)


def generate(llm, prompt_ids: list[list[int]], gen: int, batch: int | None = None):
    """Greedy decode; ``batch`` splits the prompts into engine calls of that size."""
    from vllm import SamplingParams
    from vllm.inputs import TokensPrompt

    sp = SamplingParams(temperature=0.0, max_tokens=gen, ignore_eos=True, detokenize=False)
    outs = []
    step = batch or len(prompt_ids)
    for i in range(0, len(prompt_ids), step):
        res = llm.generate([TokensPrompt(prompt_token_ids=p) for p in prompt_ids[i:i + step]], sp,
                           use_tqdm=False)
        outs.extend(list(r.outputs[0].token_ids) for r in res)
    return outs


def _timed(fn, *a):
    t0 = time.perf_counter()
    fn(*a)
    return time.perf_counter() - t0


def streams_sha(streams) -> str:
    import hashlib

    return hashlib.sha256(json.dumps(streams).encode()).hexdigest()[:16]


def _tp_list(args) -> None:
    """Run one fresh process per TP degree of ``--tp-list`` (vLLM engines do
    not release their GPUs within a process), collect decode tok/s and the
    greedy streams of each, and report whether every degree produced the
    same streams (and the same as ``--ref-streams`` when given)."""
    import subprocess
    import tempfile

    rows, streams = [], {}
    ref = None
    if args.ref_streams:
        with open(args.ref_streams) as f:
            ref = json.load(f)
    for tp in [int(x) for x in args.tp_list.split(",")]:
        out = os.path.join(tempfile.gettempdir(), f"fxpr_streams_tp{tp}.json")
        cmd = [sys.executable, "-m", "fxpr_vllm.e2e", "--preset", args.preset, "--prompts",
               str(args.prompts), "--prompt-len", str(args.prompt_len), "--gen", str(args.gen),
               "--tp", str(tp), "--out", out]
        if args.model_dir:
            cmd += ["--model-dir", args.model_dir]
        if args.eager:
            cmd += ["--eager"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if r.returncode != 0 or not line:
            rows.append({"tp": tp, "error": (r.stderr or r.stdout)[-2000:]})
            continue
        res = json.loads(line[-1])
        with open(out) as f:
            streams[tp] = json.load(f)
        res["streams_sha256_16"] = streams_sha(streams[tp])
        rows.append(res)
        print(json.dumps(res), flush=True)
    vals = list(streams.values()) + ([ref] if ref is not None else [])
    summary = {"preset": args.preset, "tp_degrees": [r["tp"] for r in rows],
               "identical_across_tp": bool(vals) and all(v == vals[0] for v in vals),
               "reference_streams_sha256_16": streams_sha(ref) if ref is not None else None,
               "runs": rows}
    print(json.dumps(summary), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="llama1b", choices=sorted(PRESETS))
    ap.add_argument("--model-dir", default=None)
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--batches", default="", help="comma list of batch sizes to compare")
    ap.add_argument("--out", default=None, help="write token streams (json) here")
    ap.add_argument("--tp-list", default="", help="comma list of TP degrees, one process each")
    ap.add_argument("--eager", action="store_true", help="no torch.compile / CUDA graphs")
    ap.add_argument("--ref-streams", default=None, help="streams (json) every TP degree must match")
    args = ap.parse_args()
    if args.tp_list:
        _tp_list(args)
        return
    d = make_llama_dir(args.model_dir or f"/tmp/fxpr_{args.preset}", args.preset)
    llm = make_llm(d, tp=args.tp, max_num_seqs=max(args.prompts, 1),
                   max_model_len=args.prompt_len + args.gen + 16, enforce_eager=args.eager)
    ps = prompts(args.prompts, args.prompt_len, PRESETS[args.preset]["vocab_size"])
    generate(llm, ps[:2], 4)  # warm-up
    generate(llm, ps, 2)      # warm-up at full batch (prefix cache off, see make_llm)
    # decode time = time(gen tokens) - time(1 token): both runs do the same prefill
    t_prefill = min(_timed(generate, llm, ps, 1) for _ in range(2))
    t_all, out = float("inf"), None
    for _ in range(2):
        t0 = time.perf_counter()
        out = generate(llm, ps, args.gen)
        t_all = min(t_all, time.perf_counter() - t0)
    decode_s = max(t_all - t_prefill, 1e-9)
    res = {"preset": args.preset, "tp": args.tp, "prompts": args.prompts,
           "prompt_len": args.prompt_len, "gen": args.gen,
           "eager": args.eager, "decode_tok_s": round(args.prompts * (args.gen - 1) / decode_s, 2),
           "total_s": round(t_all, 3), "prefill_s": round(t_prefill, 3),
           "streams_sha256_16": streams_sha(out)}
    if args.batches:
        same = True
        for b in [int(x) for x in args.batches.split(",")]:
            same &= generate(llm, ps, args.gen, batch=b) == out
        res["identical_across_batches"] = same
    if args.out:
        with open(args.out, "w") as f:
            json.dump(out, f)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
