"""Benchmark of the FxPR fixed-point reduction hot path on B200.

One *step* is one pass of the decode-time hot path over one synthetic batch,
the three op-level benchmark configurations back to back on one stream:

  1. fixed-point GEMM   A[64,4096] x W[4096,4096] bf16, Q15.16, int32      (config 1)
  2. fixed-point RMSNorm x[8192,4096] bf16 (int32) + fixed-point row sum  (config 2)
  3. paged decode attention B=64, 32/8 heads, D=128, ctx U[512,8192],
     block 16, random block permutation of a 40k-block pool, 8 KV splits  (config 3)

metric = algorithmic HBM bytes of the step / step time (GB/s), whole job
(N GPUs run N independent shards: weak scaling, no collective).
Inputs (1.3 GB per step) are larger than the 126 MB L2, so no explicit flush.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's own CPU implementation of the
path (the reference is Triton-on-GPU plus one torch CPU path; the oracle
port stands in where it has none) on the host cores, same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "fixed-point-reductions-for-vllm_b200")
for _p in (ROOT, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "fxp GEMM/attn HBM GB/s (% peak); deterministic decode tok/s at TP=1/2/4/8"
WORKLOAD = "decode_ops: gemm 64x4096x4096 + rms_norm/sum 8192x4096 + paged_attn B64 H32/8 D128 ctx512-8192"
FRAC, BITS = 16, 32


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- workload
def gemm_inputs(seed: int = 0):
    """GEMM config: A[64,4096] N(0,1), W[4096,4096] N(0,0.02), fp32 draws then bf16."""
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    W = (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)
    return dict(A=A, W=W)


def norm_inputs(seed: int = 1):
    """RMSNorm + sum config: x[8192,4096] N(0,1), w[4096] N(1,0.1)."""
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(8192, 4096, generator=g).to(torch.bfloat16)
    Wn = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    return dict(X=X, Wn=Wn)


def attention_inputs(seed: int = 2, batch: int = 64, heads: int = 32, kv_heads: int = 8,
                     head_dim: int = 128, pool: int = 40000, ctx_lo: int = 512, ctx_hi: int = 8192):
    """Paged decode attention config: per-request context U[512, 8192], page 16,
    block tables a random permutation of a 40k-block pool, q and the cache N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (batch,), generator=g)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    nblk = (ctx + 15) // 16
    bt = torch.zeros(batch, (ctx_hi + 15) // 16, dtype=torch.int32)
    off = 0
    for r in range(batch):
        n = int(nblk[r])
        bt[r, :n] = perm[off:off + n]
        off += n
    Q = torch.randn(batch, heads, head_dim, generator=g).to(torch.bfloat16)
    KV = torch.empty(pool, 2, 16, kv_heads, head_dim, dtype=torch.bfloat16)
    for i in range(0, pool, 2000):  # chunked draw to bound host memory
        KV[i:i + 2000] = torch.randn(min(2000, pool - i), 2, 16, kv_heads, head_dim,
                                     generator=g).to(torch.bfloat16)
    qsl = torch.arange(batch + 1, dtype=torch.int32)
    return dict(Q=Q, KV=KV, bt=bt, seq_lens=ctx.to(torch.int32), qsl=qsl)


def make_inputs(seed_base: int = 0):
    """CPU tensors of the three op-level configs (fp32 draws then bf16)."""
    return {**gemm_inputs(seed_base + 0), **norm_inputs(seed_base + 1),
            **attention_inputs(seed_base + 2)}


def algorithmic_bytes(inp) -> dict:
    """Bytes each op must move at minimum (read inputs once, write outputs once)."""
    M, K = inp["A"].shape
    N = inp["W"].shape[0]
    gemm = 2 * N * K + 2 * M * K + 4 * M * N
    rows, hid = inp["X"].shape
    rms = 2 * rows * hid * 2 + 2 * hid
    fsum = 2 * rows * hid + 4 * rows  # separate op: re-reads x
    sctx = int(inp["seq_lens"].sum())
    attn = sctx * 8 * 128 * 2 * 2 + sctx // 16 * 4 + 64 * 32 * 128 * 2 * 2 + 64 * 4 * 2
    return dict(gemm=gemm, rms_norm=rms, fxp_sum=fsum, attention=attn)


class Step:
    """Device-resident inputs and one launch of each hot-path kernel."""

    def __init__(self, inp, device):
        from fxpr_vllm import library_ops  # noqa: F401  (registers fxpr::*)

        self.d = {k: v.to(device) for k, v in inp.items()}
        self.y = torch.empty_like(self.d["X"])
        self.o = torch.empty_like(self.d["Q"])
        self.max_seq = int(inp["seq_lens"].max())

    def gemm(self):
        return torch.ops.fxpr.gemm_fxp(self.d["A"], self.d["W"].t(), FRAC, BITS)

    def rms(self):
        from fxpr_vllm.fixed_point_kernels import rms_norm as R

        R.rms_norm_fxp(self.d["X"], self.d["Wn"], 1e-6, FRAC, BITS, out=self.y)

    def fsum(self):
        from fxpr_vllm.fixed_point_kernels import fixed_point as F

        return F.fxp_sum(self.d["X"], FRAC, BITS)

    def attn(self):
        from fxpr_vllm.fixed_point_kernels import attention as A

        A.unified_attention_fxp(self.d["Q"], self.d["KV"], self.o, self.d["qsl"], self.d["seq_lens"],
                                self.d["bt"], 1, fxp_dtype=BITS, frac_bits=FRAC, num_kv_splits=8,
                                max_seq_len=self.max_seq)

    OPS = ("gemm", "rms_norm", "fxp_sum", "attention")

    def run(self, ev=None):
        fns = (self.gemm, self.rms, self.fsum, self.attn)
        if ev is None:
            for fn in fns:
                fn()
            return
        for i, fn in enumerate(fns):
            ev[i].record()
            fn()
        ev[len(fns)].record()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU arm
def cpu_sample(threads: int):
    """Bounded sample of the same workload through the reference's CPU path:
    the RMSNorm is the reference's own torch CPU implementation
    (``_det_norm_torch``); GEMM, sum and attention have no CPU path in the
    reference, so the oracle port stands in. Returns (GB/s, seconds, text)."""
    from oracle import fxp_oracle as O

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    A = torch.randn(64, 512, generator=g).to(torch.bfloat16)
    W = (torch.randn(4096, 512, generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(1024, 4096, generator=g).to(torch.bfloat16)
    Wn = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    from tests.helpers import paged_inputs

    q, kv, qsl, sl, bt = paged_inputs([1, 1], [4352, 4352], 32, 8, 128, 16, seed=2)
    nbytes = (2 * 4096 * 512 + 2 * 64 * 512 + 4 * 64 * 4096) + (2 * 1024 * 4096 * 2 + 8192) \
        + (2 * 1024 * 4096 + 4096) + (2 * 4352 * 8 * 128 * 2 * 2)
    t0 = time.perf_counter()
    O.gemm_fxp(A, W.t(), FRAC, BITS)
    O.rms_norm_det_torch(X.to(torch.float32), Wn, 1e-6, FRAC, BITS).to(torch.bfloat16)
    O.fxp_sum(X, FRAC, BITS)
    O.unified_attention_fxp(q, kv, torch.zeros(q.shape), qsl, sl, bt, 1, int_bits=BITS, frac_bits=FRAC)
    dt = time.perf_counter() - t0
    sample = ("gemm 64x512x4096, rms_norm(_det_norm_torch)+sum 1024x4096, "
              "paged attention 2 seqs x 4352 keys, H32/8 D128")
    return nbytes / dt / 1e9, dt, sample


# ---------------------------------------------------------------- ncu traffic
def _ncu_traffic(path):
    """DRAM bytes per attention call from an ncu CSV of this workload (sum of
    dram__bytes_read.sum + dram__bytes_write.sum over the attention kernels,
    divided by the number of calls), or None when no capture is given."""
    if not path:
        return None
    import csv

    per_kernel = {}
    with open(path) as f:
        rows = [r for r in csv.reader(line for line in f if not line.startswith("=="))]
    hdr = rows[0]
    ki, mi, vi = hdr.index("Kernel Name"), hdr.index("Metric Name"), hdr.index("Metric Value")
    for r in rows[1:]:
        if len(r) <= vi or not r[mi].startswith("dram__bytes_"):
            continue
        if "attn" not in r[ki]:
            continue
        per_kernel.setdefault(r[ki], []).append(float(r[vi].replace(",", "")))
    if not per_kernel:
        return None
    calls = min(len(v) for v in per_kernel.values()) / 2  # read + write rows per launch
    return int(sum(sum(v) for v in per_kernel.values()) / max(calls, 1))


# ---------------------------------------------------------------- main
def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return ws, rank, local


def run_reference(args, ws, rank):
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    vals, secs = [], 0.0
    for _ in range(max(args.warmup, 0)):
        cpu_sample(cores)
    sample = ""
    for _ in range(args.steps):
        v, dt, sample = cpu_sample(cores)
        vals.append(v)
        secs += dt
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1000, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32 fixed-point (Q15.16) over bf16",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample": "bounded CPU sample"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-traffic", default=None,
                    help="ncu CSV (dram__bytes_read.sum, dram__bytes_write.sum) of this workload: "
                         "fills roofline.traffic with the attention kernels' DRAM bytes per call")
    args = ap.parse_args()
    ws, rank, local = _dist()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    inp = make_inputs(seed_base=100 * rank)
    nb = algorithmic_bytes(inp)
    step_bytes = sum(nb.values())
    st = Step(inp, dev)
    for _ in range(max(args.warmup, 3)):
        st.run()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(Step.OPS) + 1)]
           for _ in range(args.steps)]
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # keep the GPU busy while the sampler starts, then time exactly K steps
        t_end = time.time() + 0.6
        while time.time() < t_end:
            st.run()
            torch.cuda.synchronize()
        start.record()
        for k in range(args.steps):
            st.run(evs[k])
        end.record()
        torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    t_ms = start.elapsed_time(end)
    per = {op: [e[i].elapsed_time(e[i + 1]) for e in evs] for i, op in enumerate(Step.OPS)}
    if ws > 1:
        tt = torch.tensor([t_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_ms = float(tt.item())
    ms_step = t_ms / args.steps
    value = step_bytes * ws / (ms_step / 1e3) / 1e9

    # e2e through the public API with host buffers (H2D inputs, D2H results)
    e2e_steps = min(args.steps, 3)
    pinned = {k: v.pin_memory() for k, v in inp.items()}
    outs_host = None
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = sum(v.numel() * v.element_size() for v in pinned.values())
    e0.record()
    for _ in range(e2e_steps):
        for k, v in pinned.items():
            st.d[k].copy_(v, non_blocking=True)
        c = st.gemm()
        st.rms()
        s = st.fsum()
        st.attn()
        outs_host = [c.to("cpu", non_blocking=True), st.y.to("cpu", non_blocking=True),
                     s.to("cpu", non_blocking=True), st.o.to("cpu", non_blocking=True)]
    e1.record()
    torch.cuda.synchronize()
    d2h = sum(t.numel() * t.element_size() for t in outs_host)
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if ws > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_val = step_bytes * ws / (e2e_ms / 1e3) / 1e9

    peak, peak_kind = _peaks()
    attn_ms = statistics.median(per["attention"])
    achieved = nb["attention"] / (attn_ms / 1e3) / 1e9
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and ws == 1:
            cores = os.cpu_count() or 1
            v, dt, sample = cpu_sample(cores)
            cpu = {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": sample + f" ({dt:.1f} s)"}
        traffic = _ncu_traffic(args.ncu_traffic)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int32 fixed-point (Q15.16) over bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "l2": "inputs 1.3 GB/step > 126 MB L2 (no flush)",
                       "parallelism": f"{ws} independent shards (weak scaling)",
                       "frac_bits": FRAC, "int_bits": BITS,
                       "algorithmic_bytes": nb,
                       "ms_per_op": {k: round(statistics.median(v), 4) for k, v in per.items()},
                       "hbm_frac_per_op": {
                           op: round(nb[op] / statistics.median(per[op]) / 1e6 / peak, 4)
                           for op in Step.OPS},
                       "gemm_products_per_s": round(64 * 4096 * 4096 / (statistics.median(per["gemm"]) / 1e3), 1)},
            "roofline": {"kernel": "paged decode attention (dq_scores + dq_pv kernels, "
                                   "2 launches per call)", "bound": "hbm",
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": 5 * args.steps,  # gemm, rms_norm, fxp_sum, 2 x attention
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
