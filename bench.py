"""Benchmark of the B200 verify-attention path (benchmark config 2 per GPU).

One step = one DSpark verify round of one layer: append 16 draft K/V (RoPE theta 1e6), verify attention
of the 16 drafts over 32768 cached tokens + drafts (split-KV + log-sum-exp combine), rollback to the
context length. value = K/V bytes the attention reads per step, all ranks, / the max-over-ranks step
time (GB/s); us_per_layer is the same time per step.

N > 1 (torchrun, one rank per GPU, NCCL): the sequence is sharded by blocks, 32768 cached tokens per
rank (weak scaling: the context is 32768 x N); the last rank also holds the drafts. Each rank computes its
shard's log-sum-exp partial, the partials are all-gathered over NVLink (NCCL) and merged by the combine
kernel on every rank.

--impl reference: the reference arithmetic restated on the host cores (the C++ oracle, OpenMP over all
threads; the reference's own Go/HIP code cannot run here), same config and metric, rank 0 only.
"""
from __future__ import annotations

import argparse
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
CTX = 32768
M = 16
QH, KVH, D = 32, 8, 64
SEED = 1
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=12)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--load-seconds", type=float, default=2.0, help="untimed replays while the clock sampler runs")
    return ap.parse_args()


def kv_bytes(tokens: int) -> int:
    return tokens * KVH * D * 2 * 2


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


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
def cpu_verify_sample(case, budget_s: float = 8.0, max_calls: int = 20):
    """The oracle (reference arithmetic restated on the host cores) on the config-2 inputs: full verify
    rounds of one layer, repeated until budget_s passes. Returns (seconds per layer, calls, threads)."""
    import numpy as np

    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    table = orc.rope_table(1e6, 1.0, D, CTX + M)
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], CTX, rope=table)
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    splits = 37
    orc.verify(case["Q"], K, V, CTX, splits=splits)   # warm-up
    calls, t0 = 0, time.perf_counter()
    while calls < max_calls:
        orc.kv_append_f16(case["newK"], case["newV"], CTX, rope=table)
        orc.verify(case["Q"], K, V, CTX, splits=splits)
        calls += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return (time.perf_counter() - t0) / calls, calls, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import synth

    case = synth.verify_case(SEED, CTX, M)
    sec, calls, threads = cpu_verify_sample(case)
    bytes_step = kv_bytes(CTX + M)
    gbs = bytes_step / sec / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": calls,
        "warmup": 1,
        "ms_per_step": round(sec * 1e3, 3),
        "us_per_layer": round(sec * 1e6, 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 softmax / fp16 P (host port)",
        "data": "synthetic (splitmix64 + Box-Muller, seed 1)",
        "config": {"workload": "config 2: verify attention, 32768 cached tokens, 16 drafts, GQA 32/8, head_dim 64",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{calls} full verify rounds of one layer (append + attention + combine)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
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

    last = rank == world - 1
    case = synth.verify_case(SEED + rank, CTX, M)   # this rank's shard of the context; drafts/Q on every rank
    if world > 1:
        # every rank uses the same drafts and queries (those of rank world - 1's stream), as one sequence would
        ref_case = synth.verify_case(SEED + world - 1, CTX, M)
        case["newK"], case["newV"], case["Q"] = ref_case["newK"], ref_case["newV"], ref_case["Q"]
    kv_begin = rank * CTX
    ctx_len = world * CTX              # global context length before the drafts
    bytes_rank = kv_bytes(CTX + (M if last else 0))
    bytes_step = kv_bytes(world * CTX + M)

    # Rotating layer caches: consecutive steps read different memory, more than the L2 in total.
    n_layers = max(2, math.ceil(3 * L2_BYTES / kv_bytes(CTX)))
    rope_np = la.rope_table(1e6, 1.0, D, ctx_len + M + 1)
    rope = torch.from_numpy(rope_np.view(np.float16)).to(dev)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    K0, V0 = t(case["K"]), t(case["V"])
    caches = []
    for _ in range(n_layers):
        blocks_total = (ctx_len + M + 64) // 32 + 1
        table = torch.zeros(blocks_total, dtype=torch.int32, device=dev)
        first_blk = kv_begin // 32
        local_blocks = (CTX + (M + 64 if last else 0)) // 32 + 1
        table[first_blk:first_blk + local_blocks] = torch.arange(local_blocks, dtype=torch.int32, device=dev)
        c = la.LayerCache(la.MODE_F16, KVH, D, ctx_len + M + 64, device=dev, block_table=table, pool_blocks=local_blocks)
        c.append(K0, V0, kv_begin)
        caches.append(c)
    del K0, V0
    q = t(case["Q"])
    nk, nv = t(case["newK"]), t(case["newV"])
    out = torch.empty_like(q)
    splits = la.verify_splits(caches[0].layout, CTX, M, 0)
    ws = torch.empty(la.lib().lfm3a_verify_workspace_bytes(M, QH, D, splits), dtype=torch.uint8, device=dev)
    part = torch.empty((M * QH, D + 2), dtype=torch.float32, device=dev)
    gathered = torch.empty((world, M * QH, D + 2), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    kernel_events = []

    def step(c, timing=None):
        """One verify round of one layer (kernels: append with the int8 V of its block, verify, combine;
        rollback adds none at a 64-aligned length)."""
        if last:
            c.append(nk, nv, ctx_len, rope=rope)
        if timing is not None:
            timing[0].record()
        if world == 1:
            c.verify(q, ctx_len, out=out, workspace=ws, splits=splits)
        else:
            end = kv_begin + CTX + (M if last else 0)
            c.verify_partial(q, kv_begin, end, ctx_len, out=part, workspace=ws, splits=splits)
        if timing is not None:
            timing[1].record()
        if world > 1:
            pg.all_gather_into_tensor(gathered, part)
            la.combine(gathered, M * QH, world, D, split_stride=M * QH * (D + 2), row_stride=D + 2, out=out.view(M * QH, D))
        if last:
            c.truncate(ctx_len)

    launches_per_step = (1 if last else 0) + (2 if splits > 1 else 1) + (1 if world > 1 else 0)

    # Warm-up (eager), then capture the timed graph with per-step kernel events.
    for i in range(max(args.warmup, 3)):
        step(caches[i % n_layers])
    torch.cuda.synchronize()
    la.sync()
    K = args.steps
    stream = torch.cuda.Stream(device=dev)
    graph = torch.cuda.CUDAGraph()
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(K)]
    with torch.cuda.graph(graph, stream=stream):
        for i in range(K):
            step(caches[i % n_layers], evs[i])
    load_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(load_graph, stream=stream):
        for i in range(n_layers * 20):
            step(caches[i % n_layers])
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    t_end = time.time() + args.load_seconds
    while time.time() < t_end:
        load_graph.replay()
        torch.cuda.synchronize()
    graph.replay()   # one more warm replay of the timed graph itself
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
    kern_ms = [a.elapsed_time(b) for a, b in evs]
    la.sync()

    # ---- e2e: the public API with host buffers, one step at a time, copies and the result read included
    e2e_steps = min(K, 200)
    hq = torch.from_numpy(np.ascontiguousarray(case["Q"])).pin_memory()
    hk = torch.from_numpy(np.ascontiguousarray(case["newK"])).pin_memory()
    hv = torch.from_numpy(np.ascontiguousarray(case["newV"])).pin_memory()
    hout = torch.empty(q.shape, dtype=torch.float16).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(nk), torch.empty_like(nv)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(e2e_steps):
        c = caches[i % n_layers]
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        if last:
            c.append(dk, dv, ctx_len, rope=rope)
        if world == 1:
            c.verify(dq, ctx_len, out=out, workspace=ws, splits=splits)
        else:
            end = kv_begin + CTX + (M if last else 0)
            c.verify_partial(dq, kv_begin, end, ctx_len, out=part, workspace=ws, splits=splits)
            pg.all_gather_into_tensor(gathered, part)
            la.combine(gathered, M * QH, world, D, split_stride=M * QH * (D + 2), row_stride=D + 2, out=out.view(M * QH, D))
        if last:
            c.truncate(ctx_len)
        hout.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    s1.record()
    torch.cuda.synchronize()
    e2e_wall = (time.perf_counter() - w0) / e2e_steps
    e2e_ms = s0.elapsed_time(s1) / e2e_steps
    la.sync()

    # max over ranks
    stats = torch.tensor([total_ms, statistics.mean(kern_ms), e2e_ms, e2e_wall * 1e3], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(stats, op=pg.ReduceOp.MAX)
    total_ms, kern_avg_ms, e2e_ms, e2e_wall_ms = stats.tolist()
    ms_step = total_ms / K

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, calls, threads = cpu_verify_sample(case)
        cpu = {"value": round(kv_bytes(CTX + M) / sec / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{calls} full verify rounds of one layer at config 2 (oracle, {threads} threads, "
                         f"{sec * 1e3:.1f} ms each)"}

    if rank == 0:
        pk = peaks()
        achieved = bytes_rank / (kern_avg_ms * 1e-3) / 1e9
        traffic = ncu_traffic("verify_m64_kernel_c2.txt") if world == 1 else None
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
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp16 (fp32 accumulation)",
            "data": "synthetic (splitmix64 + Box-Muller fp16, seed 1 + rank)",
            "config": {
                "workload": "config 2: verify round of one layer (append 16 drafts with RoPE, verify attention of 16 "
                            "tokens over 32768 cached + drafts, rollback), GQA 32/8, head_dim 64, fp16 KV"
                            + (f"; sequence sharded over {world} GPUs, 32768 cached tokens each" if world > 1 else ""),
                "context_tokens": ctx_len,
                "drafts": M,
                "splits_per_gpu": splits,
                "l2": f"{n_layers} rotating layer caches of {kv_bytes(CTX) >> 20} MiB (> 126 MB L2), no flush",
                "parallelism": f"sequence-shard x{world}" if world > 1 else "single GPU",
                "graph": "each timed step replayed from one CUDA graph of K steps",
            },
            "roofline": {
                "kernel": "verify_m64_kernel" + (" (+ per-rank partial)" if world > 1 else " + combine_kernel"),
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4),
                "peak_src": pk["src"],
                "traffic": traffic,
                "algorithmic_bytes_per_launch": bytes_rank,
                "avg_launch_us": round(kern_avg_ms * 1e3, 3),
            },
            "cpu_baseline": cpu,
            "e2e": {"value": round(bytes_step / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "us_per_layer": round(e2e_ms * 1e3, 2), "wall_us_per_layer": round(e2e_wall_ms * 1e3, 2),
                    "h2d_bytes_per_step": int(hq.numel() * 2 + hk.numel() * 2 + hv.numel() * 2),
                    "d2h_bytes_per_step": int(hout.numel() * 2),
                    "how": "LayerCache.append/verify/truncate via ctypes, pinned-host copies, stream sync per step"},
            "gpu_launches": int(launches_per_step * K),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph, load_graph
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
