"""Benchmark of the B200 verify-attention path: benchmark config 3, strong scaling over the GPUs.

One step = one DSpark verify round of one layer: append the 16 drafts' K/V (RoPE theta 1e6), verify
attention of the 16 drafts over 131072 cached tokens + drafts (split-KV + log-sum-exp merge), roll back to
the context length. value = the K/V bytes the round reads (131088 x 8 kv heads x 64 x 2 x 2, whatever the
number of GPUs) / the max-over-ranks step time (GB/s); us_per_layer is the same time per step.

N > 1 (torchrun, one rank per GPU, NCCL): the same 131072-token layer is sharded (strong scaling). Heads plan
(default): rank r holds kv heads [8r/N, 8(r+1)/N) of the whole sequence, runs its round on them, and the
outputs are exchanged (the combine's NVLink peer stores with a flag in every word, or --exchange nccl: an NCCL
all-gather). Seq plan: rank r holds a run of
64-token blocks of all heads, the last rank also the drafts; the log-sum-exp partials are all-gathered and
merged. After the timed region rank 0 checks the exchanged output against a one-GPU round of all 8 heads.

--impl reference: the reference arithmetic restated on the host cores (the C++ oracle, OpenMP over all
threads; the reference's own Go/HIP code cannot run here), same config and metric, rank 0 only; each step is
a bounded sample of the round (one kv head's share, the heads in turn).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = ROOT / "lfm3-1.7b-mi50_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "verify-attn µs/layer & HBM GB/s at 32k/128k ctx; prefill-attn int8 TOPS"
CTX3, SEED3 = 131072, 2   # config 3: the headline, on 1 GPU and sharded over N
CTX, SEED = 32768, 1      # config 2: an extra field on one GPU
M = 16
QH, KVH, D = 32, 8, 64
WORKLOAD = ("config 3: verify round of one layer (append 16 drafts with RoPE, verify attention of 16 tokens over "
            "131072 cached + drafts, rollback), GQA 32/8, head_dim 64, fp16 KV")
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=12)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--load-seconds", type=float, default=2.0, help="untimed replays while the clock sampler runs")
    ap.add_argument("--shard", choices=["heads", "seq"], default="heads", help="multi-GPU plan (N > 1)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="heads plan: NCCL all-gather of the outputs, or the combine's scatter over NVLink peer "
                         "stores with the call's flag in every word and the bounded wait kernel")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 2/4/5 and decode fields (N = 1)")
    ap.add_argument("--only", choices=["c2", "c4", "c5", "decode", "chunks", "gemm", "ref"],
                    help="run only that configuration's measurement on one GPU and print its fields (for profiling)")
    return ap.parse_args()


def run_only(args) -> int:
    import torch

    import lfm3attn as la
    import synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk = peaks()
    if args.only == "c2":
        res = measure_verify_cfg(la, synth, dev, pk["hbm_gbs"], CTX, SEED, "config 2")
    elif args.only == "c4":
        res = measure_c4(la, synth, dev, pk)
    elif args.only == "decode":
        res = measure_decodes(la, synth, dev, pk["hbm_gbs"])
    elif args.only == "chunks":
        res = measure_prefill_chunks(la, dev)
    elif args.only == "gemm":
        res = measure_gemm(la, dev, pk)
    elif args.only == "ref":
        res = measure_ref_geometries(la, synth, dev, pk["hbm_gbs"])
    else:
        res = measure_c5(la, dev)
    print(json.dumps({args.only: res}), flush=True)
    return 0


def kv_bytes(tokens: int) -> int:
    return tokens * KVH * D * 2 * 2


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p.get("bf16_tflops") or 1590.0), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def ncu_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/*.txt), else None."""
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].split()[0]))
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = pathlib.Path(f"/tmp/lfm3a_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [r for r in rows if r[4] not in ("", "[N/A]") and float(r[4]) > 0] or rows
        sm = [float(r[1]) for r in busy]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i in range(4) if r[6 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples_under_load": len(busy)}


# ------------------------------------------------------------------ CPU arm
class CpuRound:
    """The oracle (the reference arithmetic restated on the host cores, OpenMP over all threads) on config 3's
    inputs, one kv head's share of the round per step, the heads in turn: the drafts' append (RoPE) and the
    split-KV verify of its 4 query heads over 131072 cached tokens + drafts, with the combine. A step is a
    bounded sample (1/8) of the GPU arm's round."""

    def __init__(self):
        import numpy as np

        import synth
        from oracle import oracle as orc

        self.orc = orc
        self.threads = os.cpu_count() or 1
        orc.set_threads(self.threads)
        self.rope = orc.rope_table(1e6, 1.0, D, CTX3 + M)
        self.heads = []
        for h in range(KVH):
            c = synth.verify_case_heads(SEED3, CTX3, M, h, h + 1)
            k_new, v_new = orc.kv_append_f16(c["newK"], c["newV"], CTX3, rope=self.rope)
            K = np.ascontiguousarray(np.concatenate([c["K"], k_new]))
            V = np.ascontiguousarray(np.concatenate([c["V"], v_new]))
            self.heads.append((c, K, V))
        self.calls = 0

    def step(self):
        c, K, V = self.heads[self.calls % KVH]
        self.orc.kv_append_f16(c["newK"], c["newV"], CTX3, rope=self.rope)
        self.orc.verify(c["Q"], K, V, CTX3, splits=37)
        self.calls += 1

    @staticmethod
    def bytes_per_step() -> int:
        return (CTX3 + M) * D * 2 * 2   # one kv head's K and V


def cpu_baseline_sample(budget_s: float = 10.0, max_calls: int = 64) -> dict:
    """cpu_baseline of the GPU arm's line: CpuRound steps until budget_s passes."""
    r = CpuRound()
    r.step()   # warm-up
    calls, t0 = 0, time.perf_counter()
    while calls < max_calls:
        r.step()
        calls += 1
        if time.perf_counter() - t0 > budget_s:
            break
    sec = (time.perf_counter() - t0) / calls
    return {"value": round(r.bytes_per_step() / sec / 1e9, 3), "unit": "GB/s", "cores": r.threads, "kind": "port",
            "sample": f"{calls} steps of one kv head's share of the config-3 round (append + split-KV verify + "
                      f"combine of 4 query heads over 131088 keys; oracle, {r.threads} threads, "
                      f"{sec * 1e3:.1f} ms each)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    r = CpuRound()
    for _ in range(args.warmup):
        r.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r.step()
    sec = (time.perf_counter() - t0) / max(args.steps, 1)
    gbs = r.bytes_per_step() / sec / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3),
        "us_per_layer": round(sec * KVH * 1e6, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 softmax / fp16 P (host port)",
        "data": "synthetic (splitmix64 + Box-Muller fp16, seed 2)",
        "config": {"workload": WORKLOAD, "context_tokens": CTX3, "drafts": M,
                   "parallelism": f"host threads ({r.threads})",
                   "sample": "each step one kv head's share of the round (1/8 of its bytes), the heads in turn; "
                             "us_per_layer = 8 steps"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": r.threads, "kind": "port",
                         "sample": f"{args.steps} steps of one kv head's share of the config-3 round (append + "
                                   "split-KV verify + combine over 131088 keys)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
class Rank:
    """This process's share of the config-3 layer under the chosen plan (one process per GPU; strong scaling:
    the layer is the same 131072 tokens x 8 kv heads for every N).

    single  one GPU: all 8 kv heads, the 16 drafts and all 32 query heads.
    heads   rank r holds kv heads [8r/N, 8(r+1)/N) of the whole sequence and their query heads, appends its
            heads' drafts, verifies them, and the outputs are exchanged.
    seq     rank r holds a run of 64-token blocks of all heads, the last rank also the drafts; the log-sum-exp
            partials are all-gathered and merged on every rank."""

    def __init__(self, world: int, rank: int, plan: str):
        from shard import head_range, query_head_range, seq_range

        self.world, self.rank, self.plan = world, rank, plan
        self.ctx_len = CTX3
        self.kvh, self.qh = KVH, QH
        self.h0, self.h1, self.q0, self.q1 = 0, KVH, 0, QH
        self.kv_begin, self.kv_end = 0, self.ctx_len + M
        if plan == "heads":
            self.h0, self.h1 = head_range(world, rank, KVH)
            self.q0, self.q1 = query_head_range(world, rank, KVH, QH)
            self.kvh, self.qh = self.h1 - self.h0, self.q1 - self.q0
        elif plan == "seq":
            self.kv_begin, self.kv_end = seq_range(world, rank, self.ctx_len, M)
        self.drafts = plan != "seq" or rank == world - 1
        self.cached = min(self.kv_end, self.ctx_len) - self.kv_begin   # context tokens this rank holds

    def bytes_read(self) -> int:
        """K/V bytes this rank's attention reads per step."""
        return (self.kv_end - self.kv_begin) * self.kvh * D * 2 * 2


def back_to_back_us(torch, fn, n_calls: int, reps: int = 3) -> float:
    """Average device time of fn(i) over a graph of n_calls consecutive calls, events only around the graph
    (as an engine runs its layers: nothing between the calls, programmatic launch overlap intact)."""
    stream = torch.cuda.Stream()
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n_calls):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / n_calls)
    del g
    return best


def graph_step_us(torch, dev, step, steps: int) -> tuple[float, float]:
    """(µs per step of a graph of `steps` steps timed whole, µs of the events each step records around its
    attention call in a second graph of the same steps): event nodes between kernels cut the programmatic
    launch overlap, so the step time comes from the graph without them."""
    stream = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            step(i)
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(steps)]
    ge = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ge, stream=stream):
        for i in range(steps):
            step(i, evs[i])
    g.replay()
    ge.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ge.replay()
    torch.cuda.synchronize()
    step_us = e0.elapsed_time(e1) * 1e3 / steps
    att_us = statistics.mean(a.elapsed_time(b) for a, b in evs) * 1e3
    del g, ge
    return step_us, att_us


def measure_verify_cfg(la, synth, dev, peak_gbs: float, ctx: int, seed: int, label: str, steps: int = 60) -> dict:
    """A verify configuration on one GPU (config 2 as an extra field): rounds at ctx cached tokens, rotating
    layer caches that together exceed L2."""
    import numpy as np
    import torch

    case = synth.verify_case_heads(seed, ctx, M, 0, KVH)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    rope = t(la.rope_table(1e6, 1.0, D, ctx + M + 1).view(np.float16))
    K0, V0 = t(case["K"]), t(case["V"])
    n_caches = max(2, math.ceil(3 * L2_BYTES / kv_bytes(ctx)))
    caches = []
    for _ in range(n_caches):
        c = la.LayerCache(la.MODE_F16, KVH, D, ctx + M + 64, device=dev)
        c.append(K0, V0, 0)
        caches.append(c)
    del K0, V0
    q, nk, nv = t(case["Q"]), t(case["newK"]), t(case["newV"])
    out = torch.empty_like(q)
    splits = la.verify_splits(caches[0].layout, ctx, M, 0)
    ws = la.verify_workspace(M, QH, D, splits, dev)

    def step(c, ev=None):   # one round: the drafts' append fused into the attention call, then the rollback
        if ev:
            ev[0].record()
        c.verify_round(nk, nv, q, ctx, rope=rope, out=out, workspace=ws, splits=splits)
        if ev:
            ev[1].record()
        c.truncate(ctx)

    for i in range(2 * n_caches):
        step(caches[i % n_caches])
    torch.cuda.synchronize()
    step_us, att_us = graph_step_us(torch, dev, lambda i, ev=None: step(caches[i % n_caches], ev), steps)
    b2b_us = back_to_back_us(torch, lambda i: caches[i % n_caches].verify(q, ctx, out=out, workspace=ws, splits=splits),
                             60)
    la.sync()
    byts = kv_bytes(ctx + M)
    return {"workload": f"{label} on 1 GPU: verify round at {ctx} cached tokens, 16 drafts (seed {seed})",
            "us_per_layer": round(step_us, 2), "verify_us": round(att_us, 2), "splits": splits,
            "hbm_gbs": round(byts / (step_us * 1e-6) / 1e9, 1),
            "frac": round(byts / (step_us * 1e-6) / 1e9 / peak_gbs, 4),
            "verify_us_back_to_back": round(b2b_us, 2),
            "frac_back_to_back": round(byts / (b2b_us * 1e-6) / 1e9 / peak_gbs, 4),
            "bytes": byts, "caches": n_caches,
            "note": "us_per_layer / hbm_gbs / frac: a graph of rounds (the drafts' append fused into the attention "
                    "call, rollback) timed whole; verify_us: events around each round's attention call in a "
                    "second replay (event nodes cut the launch overlap); back_to_back: a graph of consecutive "
                    "verify calls timed whole"}


def measure_decode(la, synth, dev, peak_gbs: float, ctx: int, seed: int, n_caches: int, steps: int = 60) -> dict:
    """Decode attention (the scope table's first next row): one query token (m = 1) over ctx cached tokens, the
    same verify call with M = 1: append the token's K/V with RoPE, attend, roll back. Rotating caches keep
    the K/V reads above L2."""
    import numpy as np
    import torch

    case = synth.verify_case(seed, ctx, 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    rope = t(la.rope_table(1e6, 1.0, D, ctx + 2).view(np.float16))
    K0, V0 = t(case["K"]), t(case["V"])
    caches = []
    for _ in range(n_caches):
        c = la.LayerCache(la.MODE_F16, KVH, D, ctx + 64, device=dev)
        c.append(K0, V0, 0)
        caches.append(c)
    del K0, V0
    q, nk, nv = t(case["Q"]), t(case["newK"]), t(case["newV"])
    out = torch.empty_like(q)
    splits = la.verify_splits(caches[0].layout, ctx, 1, 0)
    ws = la.verify_workspace(1, QH, D, splits, dev)

    def step(c, ev=None):   # one round: the drafts' append fused into the attention call, then the rollback
        if ev:
            ev[0].record()
        c.verify_round(nk, nv, q, ctx, rope=rope, out=out, workspace=ws, splits=splits)
        if ev:
            ev[1].record()
        c.truncate(ctx)

    for i in range(2 * n_caches):
        step(caches[i % n_caches])
    torch.cuda.synchronize()
    step_us, att_us = graph_step_us(torch, dev, lambda i, ev=None: step(caches[i % n_caches], ev), steps)
    b2b_us = back_to_back_us(torch, lambda i: caches[i % n_caches].verify(q, ctx, out=out, workspace=ws, splits=splits),
                             60)
    la.sync()
    byts = kv_bytes(ctx + 1)
    return {"workload": f"decode: one query token over {ctx} cached tokens (seed {seed}), GQA 32/8, head_dim 64",
            "us_per_layer": round(step_us, 2), "attention_us": round(att_us, 2), "splits": splits,
            "hbm_gbs": round(byts / (att_us * 1e-6) / 1e9, 1), "frac": round(byts / (att_us * 1e-6) / 1e9 / peak_gbs, 4),
            "attention_us_back_to_back": round(b2b_us, 2),
            "frac_back_to_back": round(byts / (b2b_us * 1e-6) / 1e9 / peak_gbs, 4), "bytes": byts,
            "caches": n_caches}


# The reference's published verify timings on its MI50 (benchmarks/verify_attention.txt:11-14), M = 8 verified
# tokens at its own geometry (16/4/128); its K/V are int8 records (264 B per token and head), these fp16.
REF_MI50_VERIFY_US = {32768: 163.3, 131072: 557.3}


def measure_ref_geometry(la, synth, dev, peak_gbs: float, ctx: int, seed: int, n_caches: int, m: int = 8,
                         steps: int = 60) -> dict:
    """Verify at the reference model's own geometry: 16 query heads, 4 kv heads, head_dim 128 (RoPE theta 1e6
    over half the dims), m = 8 tokens over ctx cached tokens; rounds of append + attention + rollback, and the
    attention back to back. The published MI50 figure for the same m and context is reported beside it."""
    import numpy as np
    import torch

    qh, kvh, d = 16, 4, 128
    case = synth.verify_case(seed, ctx, m, q_heads=qh, kv_heads=kvh, head_dim=d)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    rope = t(la.rope_table(1e6, 0.5, d, ctx + m + 1).view(np.float16))
    K0, V0 = t(case["K"]), t(case["V"])
    caches = []
    for _ in range(n_caches):
        c = la.LayerCache(la.MODE_F16, kvh, d, ctx + 64, device=dev)
        c.append(K0, V0, 0)
        caches.append(c)
    del K0, V0
    q, nk, nv = t(case["Q"]), t(case["newK"]), t(case["newV"])
    out = torch.empty_like(q)
    splits = la.verify_splits(caches[0].layout, ctx, m, 0)
    ws = la.verify_workspace(m, qh, d, splits, dev)

    def step(c, ev=None):   # one round: append the drafts (its own kernel at head_dim 128), attend, roll back
        if ev:
            ev[0].record()
        c.verify_round(nk, nv, q, ctx, rope=rope, out=out, workspace=ws, splits=splits)
        if ev:
            ev[1].record()
        c.truncate(ctx)

    for i in range(2 * n_caches):
        step(caches[i % n_caches])
    torch.cuda.synchronize()
    step_us, att_us = graph_step_us(torch, dev, lambda i, ev=None: step(caches[i % n_caches], ev), steps)
    b2b_us = back_to_back_us(torch, lambda i: caches[i % n_caches].verify(q, ctx, out=out, workspace=ws, splits=splits),
                             60)
    la.sync()
    byts = (ctx + m) * kvh * d * 2 * 2
    res = {"workload": f"verify at the reference geometry 16/4/128: {m} tokens over {ctx} cached tokens (seed {seed})",
           "us_per_layer": round(step_us, 2), "attention_us_back_to_back": round(b2b_us, 2), "splits": splits,
           "hbm_gbs_back_to_back": round(byts / (b2b_us * 1e-6) / 1e9, 1),
           "frac_back_to_back": round(byts / (b2b_us * 1e-6) / 1e9 / peak_gbs, 4), "bytes": byts, "caches": n_caches}
    if ctx in REF_MI50_VERIFY_US:
        res["reference_mi50_us"] = REF_MI50_VERIFY_US[ctx]
    return res


# The reference's published prefill attention launches on its MI50 (benchmarks/prefill_attention.txt:12,19), ms.
REF_MI50_PREFILL_MS = {(2048, 0): {"exact": 1.43, "int8_pv": 0.72}, (7680, 115200): {"exact": 573.34, "int8_pv": 278.94}}


def measure_ref_prefill(la, dev, tokens: int, context: int, reps: int = 3) -> dict:
    """Prefill attention at the reference geometry (16/4/128): one launch of `tokens` query tokens over
    `context` cached tokens plus themselves, both variants; K/V/Q N(0,1) fp16 drawn on the device."""
    import torch

    qh, kvh, d = 16, 4, 128
    n = context + tokens
    g = torch.Generator(device=dev).manual_seed(13)
    cache = la.LayerCache(la.MODE_F16, kvh, d, n + 64, device=dev)
    step = 16384
    for p0 in range(0, n, step):
        c = min(step, n - p0)
        cache.append(torch.randn((c, kvh, d), generator=g, device=dev).half(),
                     torch.randn((c, kvh, d), generator=g, device=dev).half(), p0)
    q = torch.randn((tokens, qh, d), generator=g, device=dev).half()
    out = torch.empty_like(q)
    qk = 2.0 * qh * d * (tokens * context + tokens * (tokens + 1) / 2)
    res = {"workload": f"prefill attention at the reference geometry 16/4/128: {tokens} tokens over {context} cached",
           "qk_flop": qk}
    for name, exact in (("int8_pv", False), ("exact", True)):
        cache.prefill(q, context, exact=exact, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            cache.prefill(q, context, exact=exact, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms": round(ms, 3), "tflops_qk_plus_pv": round(2 * qk / (ms * 1e-3) / 1e12, 1)}
        ref = REF_MI50_PREFILL_MS.get((tokens, context))
        if ref:
            res[name]["reference_mi50_ms"] = ref[name]
    la.sync()
    del cache
    return res


def measure_ref_i8(la, synth, dev, peak_gbs: float, ctx: int, seed: int, n_caches: int, m: int = 8) -> dict:
    """The reference's own arithmetic over its own cache bytes at its geometry (16/4/128, int8 264-byte records):
    the m tokens' query quantiser and the int8-QK verify attention with its combine (lfm3a_quantize_q,
    lfm3a_verify_attention_i8), back to back over rotating caches. Beside it the reference's published MI50
    time for the same m and context, which runs this arithmetic on these bytes."""
    import numpy as np
    import torch

    qh, kvh, d = 16, 4, 128
    case = synth.verify_case(seed, ctx, m, q_heads=qh, kv_heads=kvh, head_dim=d)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    K0 = t(np.concatenate([case["K"], case["newK"]]))
    V0 = t(np.concatenate([case["V"], case["newV"]]))
    rope = t(la.rope_table(1e6, 0.5, d, ctx + m + 1).view(np.float16))
    caches = []
    for _ in range(n_caches):
        c = la.LayerCache(la.MODE_I8REC, kvh, d, ctx + m + 64, device=dev)
        c.append(K0, V0, 0, rope=rope)
        caches.append(c)
    del K0, V0
    q = t(case["Q"])
    qbuf = la.quantize_q(q)
    out = torch.empty_like(q)
    splits = la.lib().lfm3a_verify_i8_splits(ctypes.byref(caches[0].layout), ctx, m, 0, 0)
    ws = torch.empty(la.lib().lfm3a_verify_workspace_bytes(m, qh, d, splits), dtype=torch.uint8, device=dev)

    def call(i):   # the round's two calls: quantise the m tokens' queries, attend
        la.quantize_q(q, out=qbuf)
        caches[i % n_caches].verify_i8(qbuf, m, qh, ctx, out=out, workspace=ws, splits=splits)

    us = back_to_back_us(torch, call, 30)
    la.sync()
    byts = (ctx + m) * kvh * (2 * d + 8)
    res = {"workload": f"the reference's arithmetic on its int8 records, 16/4/128: {m} tokens over {ctx} cached "
                       f"(seed {seed})", "us_per_layer": round(us, 2), "splits": splits,
           "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1), "frac": round(byts / (us * 1e-6) / 1e9 / peak_gbs, 4),
           "bytes": byts, "caches": n_caches}
    if ctx in REF_MI50_VERIFY_US:
        res["reference_mi50_us"] = REF_MI50_VERIFY_US[ctx]
    return res


def measure_ref_i8_prefill(la, dev, tokens: int, context: int, reps: int = 3) -> dict:
    """The reference's own prefill arithmetic over its own cache bytes at its geometry (16/4/128, int8 264-byte
    records): the tokens' query quantiser and the int8 prefill attention with its key splits and combine
    (lfm3a_quantize_q, lfm3a_prefill_attention_i8), K/V/Q N(0,1) fp16 drawn on the device; beside it the
    reference's published MI50 time for the same launch (its int8 kernel on these bytes)."""
    import numpy as np
    import torch

    qh, kvh, d = 16, 4, 128
    n = context + tokens
    g = torch.Generator(device=dev).manual_seed(14)
    rope = torch.from_numpy(la.rope_table(1e6, 0.5, d, n + 1).view(np.float16)).to(dev)
    cache = la.LayerCache(la.MODE_I8REC, kvh, d, n + 64, device=dev)
    for p0 in range(0, n, 16384):
        c = min(16384, n - p0)
        cache.append(torch.randn((c, kvh, d), generator=g, device=dev).half(),
                     torch.randn((c, kvh, d), generator=g, device=dev).half(), p0, rope=rope)
    q = torch.randn((tokens, qh, d), generator=g, device=dev).half()
    qbuf = la.quantize_q(q)
    out = torch.empty_like(q)
    splits = la.lib().lfm3a_prefill_i8_splits(tokens, qh, context, 0, 0)
    ws = torch.empty(tokens * qh * splits * (d + 2) * 4, dtype=torch.uint8, device=dev)

    qk = 2.0 * qh * d * (tokens * context + tokens * (tokens + 1) / 2)
    res = {"workload": f"the reference's prefill arithmetic on its int8 records, 16/4/128: {tokens} tokens over "
                       f"{context} cached", "splits": splits}
    ref = REF_MI50_PREFILL_MS.get((tokens, context))
    for name, exact in (("int8_pv", False), ("exact", True)):
        def call():
            la.quantize_q(q, out=qbuf)
            cache.prefill_i8(qbuf, tokens, qh, context, out=out, workspace=ws, splits=splits, exact=exact)

        call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms": round(ms, 3), "tops_qk_plus_pv": round(2 * qk / (ms * 1e-3) / 1e12, 1)}
        if ref:
            res[name]["reference_mi50_ms"] = ref[name]
    la.sync()
    del cache
    return res


def measure_ref_geometries(la, synth, dev, peak_gbs: float) -> dict:
    import torch

    res = {"32k": measure_ref_geometry(la, synth, dev, peak_gbs, 32768, 11, 4)}
    torch.cuda.empty_cache()
    res["i8rec_32k"] = measure_ref_i8(la, synth, dev, peak_gbs, 32768, 11, 4)
    torch.cuda.empty_cache()
    res["i8rec_128k"] = measure_ref_i8(la, synth, dev, peak_gbs, 131072, 12, 2)
    torch.cuda.empty_cache()
    res["128k"] = measure_ref_geometry(la, synth, dev, peak_gbs, 131072, 12, 2)
    torch.cuda.empty_cache()
    res["prefill_2048"] = measure_ref_prefill(la, dev, 2048, 0)
    torch.cuda.empty_cache()
    res["prefill_7680_at_115200"] = measure_ref_prefill(la, dev, 7680, 115200)
    torch.cuda.empty_cache()
    res["i8rec_prefill_2048"] = measure_ref_i8_prefill(la, dev, 2048, 0)
    torch.cuda.empty_cache()
    res["i8rec_prefill_7680_at_115200"] = measure_ref_i8_prefill(la, dev, 7680, 115200)
    torch.cuda.empty_cache()
    return res


def measure_prefix(la, tokens: int = 131072, reps: int = 5) -> dict:
    """The prefix cache (host code in the library): register a prompt's blocks, then reuse them from a new
    sequence, for a 131072-token prompt (4096 blocks, every block chain-hashed each time)."""
    import numpy as np

    blocks = tokens // 32
    prompt = np.random.default_rng(5).integers(0, 65536, size=tokens + 1).astype(np.int32)
    reg_s, reuse_s = [], []
    for _ in range(reps):
        pc = la.PrefixCache(blocks + 8, 4 * blocks, 8)
        s = pc.sequence("bench")
        s.ensure(blocks - 1)
        _, ep = pc.alloc_conv()
        t0 = time.perf_counter()
        s.register(prompt, tokens, ep)
        reg_s.append(time.perf_counter() - t0)
        s.release()
        r = pc.sequence("bench")
        t0 = time.perf_counter()
        n, _ = r.reuse(prompt, window=256, align=2)
        reuse_s.append(time.perf_counter() - t0)
        assert n == tokens
        r.close()
        s.close()
        pc.close()
    reg, reuse = statistics.median(reg_s), statistics.median(reuse_s)
    return {"workload": f"prefix cache: register then reuse a {tokens}-token prompt ({blocks} blocks), host",
            "register_us": round(reg * 1e6, 1), "reuse_us": round(reuse * 1e6, 1),
            "reuse_ns_per_block": round(reuse * 1e9 / blocks, 1), "cores": 1}


def measure_prefill_chunks(la, dev, ctx: int = 131072, chunks=(64, 512), reps: int = 5) -> dict:
    """Prefill of a short chunk over a long cached context (a conversation's next turn, a prompt's last
    partial chunk): key splits (lfm3a_prefill_splits) against the unsplit launch (no workspace), both
    variants. K/V/Q N(0,1) from torch's seeded generator on the device."""
    import torch

    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    rnd = lambda *shape: torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).half()
    top = max(chunks)
    cache = la.LayerCache(la.MODE_F16, KVH, D, ctx + top + 64, device=dev)
    cache.append(rnd(ctx + top, KVH, D), rnd(ctx + top, KVH, D), 0)
    none = torch.empty(0, dtype=torch.uint8, device=dev)
    out = {}
    for t in chunks:
        q = rnd(t, QH, D)
        o = torch.empty_like(q)
        ws = torch.empty(max(1, la.lib().lfm3a_prefill_workspace_bytes(t, QH, D)), dtype=torch.uint8, device=dev)
        row = {"splits": la.lib().lfm3a_prefill_splits(t, QH, ctx, 0, 0)}
        for exact in (False, True):
            for name, w in (("split", ws), ("unsplit", none)):
                for _ in range(2):
                    cache.prefill(q, ctx, exact=exact, out=o, workspace=w)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    cache.prefill(q, ctx, exact=exact, out=o, workspace=w)
                e1.record()
                torch.cuda.synchronize()
                row[f"{'exact' if exact else 'int8'}_{name}_us"] = round(e0.elapsed_time(e1) * 1e3 / reps, 1)
        out[f"{t}x{ctx}"] = row
    la.sync()
    return {"workload": f"prefill chunks of {', '.join(map(str, chunks))} tokens over {ctx} cached tokens", **out}


def measure_ring(la, dev, live: int = 4096, m: int = M, ctx_len: int = 20000) -> dict:
    """The drafter's ring attention (dspark.hip:1070-1412 with RING): 16 drafts over a live ring of 4096
    positions (the reference's drafter ring, dspark.hip:70), the ring holding 4096 + 128 positions; calls back
    to back in a graph."""
    import numpy as np
    import torch

    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    rnd = lambda *shape: torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).half()
    ring_blocks = (live + 128) // 32
    table = torch.from_numpy(la.ring_table(ring_blocks, (ctx_len + m + 31) // 32 + 1)).to(dev)
    cache = la.LayerCache(la.MODE_F16, KVH, D, table.numel() * 32, device=dev, block_table=table,
                          pool_blocks=ring_blocks)
    for p0 in range(ctx_len - live - 64, ctx_len, 1024):
        n = min(1024, ctx_len - p0)
        cache.append(rnd(n, KVH, D), rnd(n, KVH, D), p0)
    cache.append(rnd(m, KVH, D), rnd(m, KVH, D), ctx_len)
    q, out = rnd(m, QH, D), torch.empty((m, QH, D), dtype=torch.float16, device=dev)
    splits = la.verify_splits(cache.layout, live, m, 0)
    ws = la.verify_workspace(m, QH, D, splits, dev)
    us = back_to_back_us(torch, lambda i: cache.ring_attention(q, ctx_len - live, ctx_len, out=out, workspace=ws,
                                                               splits=splits), 60)
    la.sync()
    byts = kv_bytes(live + m)
    return {"workload": f"drafter ring attention: {m} drafts over {live} live positions", "us": round(us, 2),
            "splits": splits, "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1), "bytes": byts,
            "note": "8.4 MB of K/V: it stays in L2 across back-to-back calls"}


def measure_decodes(la, synth, dev, peak_gbs: float) -> dict:
    """Decode (m = 1) at config 2's and config 3's context lengths and seeds, and the drafter's ring."""
    return {"32k": measure_decode(la, synth, dev, peak_gbs, CTX, SEED, 4),
            "128k": measure_decode(la, synth, dev, peak_gbs, 131072, 2, 2),
            "ring_4096": measure_ring(la, dev)}


def measure_c4(la, synth, dev, peaks_: dict, reps: int = 5) -> dict:
    """Config 4: causal prefill attention of 32768 tokens (seed 3), int8-PV and exact fp16."""
    import numpy as np
    import torch

    T = 32768
    case = synth.prefill_case(3, T)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    cache = la.LayerCache(la.MODE_F16, KVH, D, T + 64, device=dev)
    cache.append(t(case["K"]), t(case["V"]), 0)
    q = t(case["Q"])
    out = torch.empty_like(q)
    flops = 2.0 * QH * D * T * (T + 1) / 2   # QK; PV has the same count
    res = {"workload": "config 4: causal prefill attention, 32768 tokens, GQA 32/8, head_dim 64 (seed 3)",
           "qk_flop": flops, "pv_ops": flops}
    tf16 = peaks_.get("bf16_tflops")
    for name, exact in (("int8_pv", False), ("exact", True)):
        for _ in range(2):
            cache.prefill(q, 0, exact=exact, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            cache.prefill(q, 0, exact=exact, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        entry = {"ms": round(ms, 3), "pv_tops": round(flops / (ms * 1e-3) / 1e12, 1)}
        if tf16:
            # roofline time: QK at the fp16 (bf16-measured) dense peak, PV at the int8 peak (twice the fp16 rate)
            # or at the fp16 peak for the exact kernel
            t_roof = flops / (tf16 * 1e12) + flops / ((2.0 if not exact else 1.0) * tf16 * 1e12)
            entry["tensor_frac"] = round(t_roof / (ms * 1e-3), 4)
        res[name] = entry
    la.sync()
    if tf16:
        res["peak"] = f"{tf16} TFLOP/s dense fp16 (measured bf16), int8 at twice that (nominal ratio)"
    return res


# The prefill's W8A8 linear layers of one full-attention layer of LFM3-1.7B (H 2048, I 7680; mix 3088 outputs,
# internal/model/prefill.go:100-110,420-450), at the reference's long-prompt chunk of 7680 tokens (prefill.go:24).
GEMM_TOKENS = 7680
GEMM_LAYERS = (("mix", 3088, 2048, False), ("out", 2048, 2048, False), ("w13", 15360, 2048, False),
               ("w2", 2048, 7680, True))


def measure_gemm(la, dev, peaks_: dict, reps: int = 10) -> dict:
    """The hot-path table's fourth "next" row: per linear layer, the GEMM alone on quantised activations and the
    whole linear call (quantiser + GEMM), CUDA events over reps back-to-back calls after two warm-up calls."""
    import torch

    g = torch.Generator(device=dev).manual_seed(5)
    tf16 = peaks_.get("bf16_tflops")
    res = {"workload": f"W8A8 group-128 linear layers of one attention layer, {GEMM_TOKENS}-token chunk "
                       "(LFM3-1.7B shapes, random int8 weights)"}
    total_ops, total_ms = 0.0, 0.0
    for name, outputs, k, gated in GEMM_LAYERS:
        x = (torch.randn((GEMM_TOKENS, 2 * k if gated else k), generator=g, device=dev) * 2).half()
        w = torch.randint(-127, 128, (outputs, k), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
        ws = (torch.rand((outputs, k // 128), generator=g, device=dev) * 0.01 + 1e-3).half().float()
        b = la.G128Operand.pack(w, ws)
        del w
        a = la.G128Operand.quantize(x, k, gated=gated)
        out = torch.empty((GEMM_TOKENS, outputs), dtype=torch.float16, device=dev)
        ws_buf = torch.empty(la.g128_workspace_bytes(GEMM_TOKENS, k), dtype=torch.uint8, device=dev)
        ops = 2.0 * GEMM_TOKENS * outputs * k

        def timed(fn):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / reps

        ms_gemm = timed(lambda: la.g128_gemm(a, b, out=out))
        ms_lin = timed(lambda: la.g128_linear(x, b, gated=gated, out=out, workspace=ws_buf))
        entry = {"outputs": outputs, "k": k, "gated": gated, "gemm_us": round(ms_gemm * 1e3, 1),
                 "gemm_tops": round(ops / (ms_gemm * 1e-3) / 1e12, 1), "linear_us": round(ms_lin * 1e3, 1)}
        if tf16:
            entry["int8_frac"] = round(ops / (ms_gemm * 1e-3) / (2.0 * tf16 * 1e12), 4)
        res[name] = entry
        total_ops += ops
        total_ms += ms_lin
        del x, a, b, out, ws_buf
        torch.cuda.empty_cache()
    la.sync()
    res["layer_linear_us"] = round(total_ms * 1e3, 1)
    res["layer_tops"] = round(total_ops / (total_ms * 1e-3) / 1e12, 1)
    if tf16:
        res["peak"] = f"int8 dense at twice the measured bf16 {tf16} TFLOP/s (nominal ratio)"
    return res


def measure_c5(la, dev, layers: int = 4, ctx: int = 131072, steps: int = 256, seed: int = 4, R=None, pg=None,
               gg=None) -> dict:
    """Config 5, the KV lifecycle: per layer a causal prefill of ctx tokens (append with RoPE + int8-PV
    attention), then `steps` DSpark rounds over all layers (append 16 drafts, verify 16, keep
    n = min(16, X), X ~ geometric(0.3), roll back 16 - n). Inputs N(0,1) fp16 from torch's seeded generator
    on the device (the splitmix64 stream is too slow on the host at this size).

    On N GPUs (R: the rank's kv-head plan) every rank draws the same inputs and keeps its kv heads: its prefill
    stays local (its heads' outputs feed a row-parallel output projection), and each round's verify output is
    exchanged (gg: the peer-store exchange, else the NCCL all-gather). Times are the max over ranks."""
    import numpy as np
    import torch

    world = R.world if R is not None else 1
    h0, h1 = (R.h0, R.h1) if R is not None else (0, KVH)
    q0, q1 = (R.q0, R.q1) if R is not None else (0, QH)
    kvh, qh = h1 - h0, q1 - q0
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    rnd = lambda *shape: torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).half()
    rng = np.random.default_rng(seed)
    keep = np.minimum(16, rng.geometric(0.3, size=steps))
    cap = ctx + int(keep.sum()) + M + 64
    rope = torch.from_numpy(la.rope_table(1e6, 1.0, D, cap + 1).view(np.float16)).to(dev)
    caches = [la.LayerCache(la.MODE_F16, kvh, D, cap, device=dev) for _ in range(layers)]
    q_pre = rnd(ctx, QH, D)[:, q0:q1].contiguous()
    out_pre = torch.empty_like(q_pre)
    torch.cuda.synchronize()
    e0, e1, e2, e3 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
    k_in = [(rnd(ctx, KVH, D)[:, h0:h1].contiguous(), rnd(ctx, KVH, D)[:, h0:h1].contiguous()) for _ in range(layers)]
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0.record()
    for c, (k, v) in zip(caches, k_in):
        c.append(k, v, 0, rope=rope)
        c.prefill(q_pre, 0, exact=False, out=out_pre)
    e1.record()
    torch.cuda.synchronize()
    del k_in, q_pre, out_pre
    drafts = rnd(steps, 2, M, KVH, D)[:, :, :, h0:h1].contiguous()
    qs = rnd(steps, M, QH, D)[:, :, q0:q1].contiguous()
    ws = la.verify_workspace(M, qh, D, 2 * 148, dev)
    out = torch.empty((M, qh, D), dtype=torch.float16, device=dev)
    gathered = torch.empty((world, M, qh, D), dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    length = ctx
    with torch.cuda.graph(g, stream=stream):
        for s in range(steps):
            for c in caches:
                if gg is not None:
                    gg.verify_round(c, drafts[s, 0], drafts[s, 1], qs[s], length, rope=rope, workspace=ws)
                    gg.wait(gathered)
                else:
                    c.verify_round(drafts[s, 0], drafts[s, 1], qs[s], length, rope=rope, out=out, workspace=ws)
                    if pg:
                        pg.all_gather_into_tensor(gathered, out)
                c.truncate(length + int(keep[s]))
            length += int(keep[s])
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e2.record()
    g.replay()
    e3.record()
    torch.cuda.synchronize()
    la.sync()
    prefill_ms = e0.elapsed_time(e1)   # the prefill alone: the graph capture between e1 and e2 is host work
    verify_ms = e2.elapsed_time(e3)
    t = torch.tensor([prefill_ms, verify_ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    prefill_ms, verify_ms = t.tolist()
    lengths = sorted({c.length for c in caches})
    del g, caches
    res = {"workload": f"config 5: KV lifecycle, {layers} layers, {ctx}-token causal prefill (int8-PV), then "
                       f"{steps} rounds of 16 drafts (keep min(16, Geom(0.3)))",
           "data": "torch.randn N(0,1) fp16 on the device, seed 4; keep lengths from numpy default_rng(4)",
           "total_ms": round(prefill_ms + verify_ms, 2), "prefill_ms": round(prefill_ms, 2),
           "verify_ms": round(verify_ms, 2),
           "us_per_layer_round": round(verify_ms * 1e3 / (steps * layers), 2),
           "final_length": lengths[0] if len(lengths) == 1 else lengths, "expected_length": ctx + int(keep.sum())}
    if world > 1:
        res["parallelism"] = (f"kv-head shard x{world}: prefill local, each round's output exchanged "
                              + ("over NVLink peer stores" if gg is not None else "by NCCL all-gather") +
                              "; max over ranks")
    return res


def run_ours(args):
    import numpy as np
    import torch

    import lfm3attn as la
    import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = dist
    R = Rank(world, rank, args.shard if world > 1 else "single")

    # Inputs: config 3's stream (seed 2: K, V, new K, new V, Q); each rank draws only its kv heads (heads plan)
    # or slices its token run (seq plan), bit-identical to slicing the whole draw.
    case = synth.verify_case_heads(SEED3, CTX3, M, R.h0, R.h1)
    Kc = case["K"][R.kv_begin:R.kv_begin + R.cached]
    Vc = case["V"][R.kv_begin:R.kv_begin + R.cached]
    newK, newV, Qr = case["newK"], case["newV"], case["Q"]

    n_layers = max(2, math.ceil(3 * L2_BYTES / (R.cached * R.kvh * D * 4)))
    rope_np = la.rope_table(1e6, 1.0, D, R.ctx_len + M + 1)
    rope = torch.from_numpy(rope_np.view(np.float16)).to(dev)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    K0, V0 = t(Kc), t(Vc)
    del Kc, Vc
    caches = []
    cap = R.ctx_len + M + 64
    for _ in range(n_layers):
        table = torch.zeros((cap + 31) // 32, dtype=torch.int32, device=dev)
        lb0 = R.kv_begin // 32
        local_blocks = (R.cached + (M + 64 if R.drafts else 0)) // 32 + 1
        table[lb0:lb0 + local_blocks] = torch.arange(local_blocks, dtype=torch.int32, device=dev)
        c = la.LayerCache(la.MODE_F16, R.kvh, D, cap, device=dev, block_table=table, pool_blocks=local_blocks)
        c.append(K0, V0, R.kv_begin)
        caches.append(c)
    del K0, V0
    q = t(Qr)
    nk, nv = t(newK), t(newV)
    out = torch.empty((M, QH, D), dtype=torch.float16, device=dev)
    out_l = torch.empty_like(q)
    splits = la.verify_splits(caches[0].layout, R.kv_end - R.kv_begin if R.plan == "seq" else R.ctx_len, M, 0)
    ws = la.verify_workspace(M, R.qh, D, splits, dev)
    part = torch.empty((M * QH, D + 2), dtype=torch.float32, device=dev)
    gathered = torch.empty((world, M * QH, D + 2), dtype=torch.float32, device=dev)
    gathered_out = torch.empty((world, M, R.qh, D), dtype=torch.float16, device=dev)
    gg = None
    if R.plan == "heads" and args.exchange == "p2p":
        def exchange(handle):
            handles = [None] * world
            pg.all_gather_object(handles, handle)
            return handles

        gg = la.GatherGroup(world, rank, M * R.qh, D, exchange=exchange)
    torch.cuda.synchronize()

    # The single-GPU and kv-head plans run each round's append and attention as one call (lfm3a_verify_round:
    # the drafts' append fused into the attention kernel); the others append first.
    fused_round = R.drafts and R.plan in ("single", "heads")

    def attend(c, dq, timing=None, dk=None, dv=None):
        if timing is not None:
            timing[0].record()
        if R.plan == "seq":
            c.verify_partial(dq, R.kv_begin, R.kv_end, R.ctx_len, out=part, workspace=ws, splits=splits)
        elif gg is not None and fused_round and dk is not None:
            gg.verify_round(c, dk, dv, dq, R.ctx_len, rope=rope, workspace=ws, splits=splits)
        elif gg is not None:
            gg.verify(c, dq, R.ctx_len, workspace=ws, splits=splits)
        elif fused_round and dk is not None:
            c.verify_round(dk, dv, dq, R.ctx_len, rope=rope, out=out_l if R.plan == "heads" else out, workspace=ws,
                           splits=splits)
        elif R.plan == "heads":
            c.verify(dq, R.ctx_len, out=out_l, workspace=ws, splits=splits)
        else:
            c.verify(dq, R.ctx_len, out=out, workspace=ws, splits=splits)
        if timing is not None:
            timing[1].record()
        if R.plan == "seq":
            pg.all_gather_into_tensor(gathered, part)
            la.combine(gathered, M * QH, world, D, split_stride=M * QH * (D + 2), row_stride=D + 2,
                       out=out.view(M * QH, D))
        elif gg is not None:
            gg.wait(gathered_out)
        elif R.plan == "heads":
            pg.all_gather_into_tensor(gathered_out, out_l)

    def step(c, timing=None, dq=None, dk=None, dv=None):
        """One verify round of one layer: the drafts' append with the int8 V of their blocks (inside the attention
        kernel on the fused plans), verify, exchange; rollback adds no kernel at a 64-aligned length."""
        dk = nk if dk is None else dk
        dv = nv if dv is None else dv
        if R.drafts and not fused_round:
            c.append(dk, dv, R.ctx_len, rope=rope)
        attend(c, q if dq is None else dq, timing, dk if R.drafts else None, dv)
        if R.drafts:
            c.truncate(R.ctx_len)

    launches_per_step = ((1 if R.drafts and not fused_round else 0) + (2 if splits > 1 else 1) +
                         (1 if R.plan == "seq" or gg else 0))

    # Warm-up (eager), then capture the timed graph (the K steps as they run) and a second graph of the same K
    # steps with CUDA events around each verify call, replayed after the timed region for the roofline's
    # per-launch duration (event nodes between kernels cut the programmatic launch overlap, so they stay out
    # of the timed graph).
    for i in range(max(args.warmup, 3)):
        step(caches[i % n_layers])
    torch.cuda.synchronize()
    la.sync()
    K = args.steps
    stream = torch.cuda.Stream(device=dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(K):
            step(caches[i % n_layers])
    kgraph = torch.cuda.CUDAGraph()
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(K)]
    with torch.cuda.graph(kgraph, stream=stream):
        for i in range(K):
            step(caches[i % n_layers], evs[i])
    load_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(load_graph, stream=stream):
        for i in range(n_layers * 20):
            step(caches[i % n_layers])
    torch.cuda.synchronize()

    # Load phase for the clock sampler. The graphs hold NCCL collectives on N > 1, so every rank must replay
    # them the same number of times: the count comes from the slowest rank's replay time, not from a clock.
    t0 = time.perf_counter()
    load_graph.replay()
    torch.cuda.synchronize()
    one = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(one, op=pg.ReduceOp.MAX)
    n_load = max(1, int(args.load_seconds / max(float(one.item()), 1e-4)))
    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(n_load):
        load_graph.replay()
        torch.cuda.synchronize()
    graph.replay()   # one more warm replay of the timed graph itself
    torch.cuda.synchronize()
    kgraph.replay()
    torch.cuda.synchronize()

    # ---- timed region: exactly K steps
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    clocks = sampler.stop()
    total_ms = e0.elapsed_time(e1)
    # The roofline's per-launch duration: the same K steps with events around each verify call.
    kgraph.replay()
    torch.cuda.synchronize()
    kern_ms = [a.elapsed_time(b) for a, b in evs]
    la.sync()
    b2b_us = None
    if world == 1:   # the verify calls alone, back to back over the same rotating caches
        b2b_us = back_to_back_us(torch, lambda i: attend(caches[i % n_layers], q), 3 * n_layers)
        la.sync()

    # ---- check: on N > 1 the exchanged output of one more eager step against a one-GPU round of all 8 heads
    # (rank 0's GPU); on one GPU the round's output is what the test suite checks against the oracle.
    check = None
    step(caches[0])
    torch.cuda.synchronize()
    la.sync()
    if world > 1 and rank == 0:
        import shard

        got = out if R.plan == "seq" else shard.assemble_heads(gathered_out)
        full = synth.verify_case_heads(SEED3, CTX3, M, 0, KVH)
        ref_cache = la.LayerCache(la.MODE_F16, KVH, D, CTX3 + M + 64, device=dev)
        ref_cache.append(t(full["K"]), t(full["V"]), 0)
        want = ref_cache.verify_round(t(full["newK"]), t(full["newV"]), t(full["Q"]), CTX3, rope=rope)
        la.sync()
        g64, w64 = got.double().cpu(), want.double().cpu()
        rms = float(w64.pow(2).mean().sqrt())
        check = {"against": "one-GPU lfm3a_verify_round of all 8 kv heads on rank 0's GPU",
                 "max_abs_err_rel_rms": float((g64 - w64).abs().max()) / rms,
                 "bit_identical": bool(torch.equal(got.cpu(), want.cpu()))}
        del ref_cache, want, full

    # ---- e2e: the public API with host buffers, one step at a time, copies and the result read included.
    # The step's inputs (the drafts' queries, keys and values) travel from one pinned host buffer in one copy.
    e2e_steps = min(K, 200)
    nq_, nk_ = q.numel(), nk.numel()
    hin = torch.empty(nq_ + 2 * nk_, dtype=torch.float16).pin_memory()
    hin[:nq_].copy_(torch.from_numpy(np.ascontiguousarray(Qr)).reshape(-1))
    hin[nq_:nq_ + nk_].copy_(torch.from_numpy(np.ascontiguousarray(newK)).reshape(-1))
    hin[nq_ + nk_:].copy_(torch.from_numpy(np.ascontiguousarray(newV)).reshape(-1))
    din = torch.empty(hin.shape, dtype=torch.float16, device=dev)
    dq = din[:nq_].view(q.shape)
    dk = din[nq_:nq_ + nk_].view(nk.shape)
    dv = din[nq_ + nk_:].view(nv.shape)
    res = gathered_out if R.plan == "heads" else out
    hout = torch.empty(res.shape, dtype=torch.float16).pin_memory()
    direct = world == 1 and fused_round
    if direct:
        # One GPU: the round with host buffers is one C-ABI call (lfm3a_verify_round_host: the drafts' copy in, the
        # round, the output's copy out, queued without waiting), then the rollback (lfm3a_kv_truncate), then one
        # stream synchronize, with the arguments prepared once, as a caller that keeps its layer views does.
        lib = la.lib()
        views = [ctypes.byref(c.view) for c in caches]
        st_ptr = torch.cuda.current_stream().cuda_stream
        ws_bytes = ws.numel()
        call_args = (hin.data_ptr(), din.data_ptr(), rope.data_ptr(), None, M, QH, R.ctx_len, 0, None, out.data_ptr(),
                     hout.data_ptr(), ws.data_ptr(), ws_bytes, splits, st_ptr, -1)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    rc_e2e = 0
    for i in range(e2e_steps):
        if direct:
            rc_e2e |= lib.lfm3a_verify_round_host(views[i % n_layers], *call_args)
            rc_e2e |= lib.lfm3a_kv_truncate(views[i % n_layers], R.ctx_len, st_ptr)
            torch.cuda.current_stream().synchronize()
        else:
            din.copy_(hin, non_blocking=True)
            step(caches[i % n_layers], None, dq, dk, dv)
            hout.copy_(res, non_blocking=True)
            torch.cuda.current_stream().synchronize()
    s1.record()
    torch.cuda.synchronize()
    if rc_e2e:
        raise la.LFM3AError(rc_e2e, "e2e round")
    e2e_wall = (time.perf_counter() - w0) / e2e_steps
    e2e_ms = s0.elapsed_time(s1) / e2e_steps
    la.sync()

    # max over ranks
    stats = torch.tensor([total_ms, statistics.mean(kern_ms), e2e_ms, e2e_wall * 1e3], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total_ms, kern_avg_ms, e2e_ms, e2e_wall_ms = stats.tolist()
    ms_step = total_ms / K
    bytes_step = kv_bytes(R.ctx_len + M)   # all ranks together

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()
    del graph, kgraph, load_graph

    extras = {}
    if world > 1 and not args.no_extras and R.plan == "heads":   # config 5 on the same plan, every rank
        del caches
        torch.cuda.empty_cache()
        extras["c5"] = measure_c5(la, dev, R=R, pg=pg, gg=gg)
    if rank == 0 and world == 1 and not args.no_extras:
        pk = peaks()
        del caches
        torch.cuda.empty_cache()
        extras["c2"] = measure_verify_cfg(la, synth, dev, pk["hbm_gbs"], CTX, SEED, "config 2")
        torch.cuda.empty_cache()
        extras["decode"] = measure_decodes(la, synth, dev, pk["hbm_gbs"])
        extras["prefix"] = measure_prefix(la)
        torch.cuda.empty_cache()
        extras["c4"] = measure_c4(la, synth, dev, pk)
        torch.cuda.empty_cache()
        extras["prefill_chunks"] = measure_prefill_chunks(la, dev)
        torch.cuda.empty_cache()
        extras["gemm"] = measure_gemm(la, dev, pk)
        torch.cuda.empty_cache()
        extras["ref_geometry"] = measure_ref_geometries(la, synth, dev, pk["hbm_gbs"])
        torch.cuda.empty_cache()
        extras["c5"] = measure_c5(la, dev)

    if rank == 0:
        pk = peaks()
        achieved = R.bytes_read() / (kern_avg_ms * 1e-3) / 1e9
        traffic = ncu_traffic("verify_m64_kernel_c3.txt") if world == 1 else None
        plan_text = {"single": "single GPU",
                     "heads": f"kv-head shard x{world}" + (", outputs over NVLink peer stores" if gg else ", NCCL all-gather"),
                     "seq": f"sequence shard x{world}, NCCL all-gather of partials"}
        line = {
            "metric": METRIC,
            "value": round(bytes_step / (ms_step * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms_step, 5),
            "us_per_layer": round(ms_step * 1e3, 2),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp16 (fp32 accumulation)",
            "data": "synthetic (splitmix64 + Box-Muller fp16, seed 2)",
            "config": {
                "workload": WORKLOAD + (f"; {plan_text[R.plan]}" if world > 1 else ""),
                "context_tokens": R.ctx_len,
                "drafts": M,
                "kv_heads_per_gpu": R.kvh,
                "tokens_per_gpu": R.kv_end - R.kv_begin,
                "splits_per_gpu": splits,
                "l2": f"{n_layers} rotating layer caches of {R.cached * R.kvh * D * 4 >> 20} MiB of K/V per GPU "
                      "(> 126 MB L2 together), no flush",
                "parallelism": plan_text[R.plan],
                "graph": "each timed step replayed from one CUDA graph of K steps",
            },
            "roofline": {
                "kernel": "verify_m64_kernel + combine_kernel" + (" (per rank)" if world > 1 else ""),
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4),
                "peak_src": pk["src"],
                "traffic": traffic,
                "algorithmic_bytes_per_launch": R.bytes_read(),
                "avg_launch_us": round(kern_avg_ms * 1e3, 3),
                "back_to_back_us": None if b2b_us is None else round(b2b_us, 3),
                "frac_back_to_back": None if b2b_us is None else round(R.bytes_read() / (b2b_us * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
                "note": "achieved / frac: CUDA events around each verify call in a replay of the timed steps "
                        "(event nodes cut the programmatic launch overlap, so the timed graph itself has none); "
                        "back_to_back: a graph of consecutive verify + combine calls over the same rotating caches, "
                        "events around the graph",
            },
            "cpu_baseline": cpu,
            "e2e": {"value": round(bytes_step / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "us_per_layer": round(e2e_ms * 1e3, 2), "wall_us_per_layer": round(e2e_wall_ms * 1e3, 2),
                    "h2d_bytes_per_step": int(hin.numel() * 2),
                    "d2h_bytes_per_step": int(hout.numel() * 2),
                    "how": ("per step lfm3a_verify_round_host (one copy of the drafts' q, k, v from pinned host "
                            "memory, the round, the output copied back to pinned host memory) + lfm3a_kv_truncate "
                            "through ctypes, then a stream synchronize" if direct else
                            "one pinned-host copy of this rank's drafts' q, k, v, the plan's step (LayerCache calls "
                            "and the exchange), the exchanged output read back, a stream sync per step")},
            "gpu_launches": int(launches_per_step * K),
            "clocks": clocks,
        }
        if check is not None:
            line["check"] = check
        line.update(extras)
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        if gg is not None:   # every rank unmaps its peers' regions before any region is freed
            gg.unmap()
            pg.barrier()
            gg.free()
        pg.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.only:
        return run_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
