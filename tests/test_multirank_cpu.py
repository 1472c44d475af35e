"""The multi-GPU plans on CPU: two gloo ranks (127.0.0.1), each computing its shard with the oracle, the
shards exchanged with all_gather as the GPU ranks exchange them over NCCL.

heads: each rank verifies its kv heads' query heads; the gathered outputs, laid side by side, equal the
       single-process oracle bit for bit.
seq:   each rank computes the partial (acc, max, sum) of its blocks; the gathered partials merged by the
       combine equal the single-process oracle within 2e-3 of the RMS (the fp16 rounding of each probability
       depends on the running max, which differs between one pass and two shards).
Also the plans themselves: contiguous, covering, aligned to the 64-token int8 V blocks, empty ranks allowed.
"""
import os
import socket

import numpy as np
import pytest

from shard import assemble_heads, head_range, query_head_range, seq_range


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plans_cover_the_sequence():
    for world in (1, 2, 3, 4, 8):
        for ctx, m in ((0, 1), (20, 4), (1000, 16), (32768 * 2, 16), (100000, 7)):
            ranges = [seq_range(world, r, ctx, m) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == ctx + m
            for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
                assert e0 == b1 and b0 <= e0
                assert b1 % 64 == 0 or b1 == ctx
    assert [head_range(4, r, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert query_head_range(2, 1, 8, 32) == (16, 32)
    with pytest.raises(ValueError):
        head_range(3, 0, 8)


def _rank_main(rank, world, port, case, mode, window, result_dir):
    import torch
    import torch.distributed as dist

    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc.set_threads(2)
        Q, K, V, ctx, gate = case["Q"], case["K"], case["V"], case["ctx"], case["gate"]
        m, qh, d = Q.shape
        kvh = K.shape[1]
        if mode == "heads":
            h0, h1 = head_range(world, rank, kvh)
            q0, q1 = query_head_range(world, rank, kvh, qh)
            g = None if gate is None else np.ascontiguousarray(gate[:, q0:q1])
            mine = orc.verify(Q[:, q0:q1], K[:, h0:h1], V[:, h0:h1], ctx, window=window, gate=g)
            parts = [torch.empty(mine.shape, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(mine))
            got = assemble_heads(torch.stack(parts)).numpy()
        else:
            b, e = seq_range(world, rank, ctx, m)
            if e > b:
                mine = orc.verify_partial(Q, K, V, b, e, ctx, window=window)
            else:   # an empty shard: weight zero in the merge
                mine = np.zeros((m * qh, d + 2), dtype=np.float32)
                mine[:, d] = -np.inf
            parts = [torch.empty(mine.shape, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(mine))
            got = orc.combine(torch.stack(parts).numpy(), d, gate=gate).reshape(m, qh, d)
        if rank == 0:
            np.save(os.path.join(result_dir, "got.npy"), got)
    finally:
        dist.destroy_process_group()


def run_ranks(world, case, mode, window, tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(world, free_port(), case, mode, window, str(tmp_path)), nprocs=world, join=True)
    return np.load(tmp_path / "got.npy")


def make_case(synth, seed, ctx, m, gate=False):
    c = synth.verify_case(seed, ctx, m)
    K = np.concatenate([c["K"], c["newK"]])
    V = np.concatenate([c["V"], c["newV"]])
    g = synth.Stream(seed + 100).normal_f16((m, 32)) if gate else None
    return {"Q": c["Q"], "K": K, "V": V, "ctx": ctx, "gate": g}


@pytest.mark.parametrize("window,gate", [(0, False), (300, True)])
def test_heads_plan_two_ranks(orc, synth, tmp_path, window, gate):
    case = make_case(synth, 40, 1500, 8, gate)
    got = run_ranks(2, case, "heads", window, tmp_path)
    want = orc.verify(case["Q"], case["K"], case["V"], case["ctx"], window=window, gate=case["gate"])
    assert np.array_equal(got, want)


@pytest.mark.parametrize("ctx,window,gate", [(1500, 0, False), (1500, 300, True), (20, 0, False)])
def test_seq_plan_two_ranks(orc, synth, tmp_path, ctx, window, gate):
    case = make_case(synth, 41, ctx, 8, gate)
    got = run_ranks(2, case, "seq", window, tmp_path)
    want = orc.verify(case["Q"], case["K"], case["V"], ctx, window=window, gate=case["gate"]).astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    assert float(np.max(np.abs(got - want))) / rms < 2e-3
