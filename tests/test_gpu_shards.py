"""The multi-GPU building blocks on one GPU: the cache split as the ranks of the two plans would hold it.

seq:   two shard caches (block tables indexed by global position, each pool holding only its own blocks)
       give lfm3a_verify_partial partials whose normalised value acc / sum matches the oracle's partial of
       the same keys, and lfm3a_combine of the two matches the oracle's whole verify.
heads: two caches of 4 kv heads each, verified separately, match the oracle's verify of all 8 heads.
Tolerance 4e-3 of the RMS beyond half an fp16 ulp for fp16 outputs, as in the verify tests.
"""
import numpy as np
import pytest

from shard import head_range, query_head_range, seq_range

pytestmark = pytest.mark.gpu

TOL_PAIR = 4e-3


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


def full_case(synth, seed, ctx, m):
    c = synth.verify_case(seed, ctx, m)
    return c["Q"], np.concatenate([c["K"], c["newK"]]), np.concatenate([c["V"], c["newV"]])


def shard_cache(la, cuda, K, V, b, e, capacity, kv_heads=8):
    import torch

    lb0, lb1 = b // 32, (e + 31) // 32
    table = torch.zeros((capacity + 31) // 32, dtype=torch.int32, device=cuda)
    table[lb0:lb1] = torch.arange(lb1 - lb0, dtype=torch.int32, device=cuda)
    cache = la.LayerCache(la.MODE_F16, kv_heads, 64, capacity, device=cuda, block_table=table, pool_blocks=lb1 - lb0)
    cache.append(dev(K[b:e], cuda), dev(V[b:e], cuda), b)
    return cache


@pytest.mark.parametrize("ctx,m,window", [(4000, 16, 0), (40000, 16, 0), (4000, 8, 1500)])
def test_seq_shards_partial_and_combine(la, orc, synth, cuda, ctx, m, window):
    import torch

    Q, K, V = full_case(synth, 50 + m, ctx, m)
    q = dev(Q, cuda)
    parts = []
    for r in range(2):
        b, e = seq_range(2, r, ctx, m)
        cache = shard_cache(la, cuda, K, V, b, e, ctx + m + 64)
        part = cache.verify_partial(q, b, e, ctx, window=window)
        la.sync()
        got = part.cpu().numpy()
        want = orc.verify_partial(Q, K, V, b, e, ctx, window=window)
        live = want[:, 65] > 0
        if live.any():
            g = got[live, :64] / got[live, 65:66]
            w = want[live, :64] / want[live, 65:66]
            assert float(np.max(np.abs(g - w))) / float(np.sqrt(np.mean(w.astype(np.float64) ** 2))) < TOL_PAIR
        parts.append(part)
    rows = m * 32
    out = la.combine(torch.stack(parts), rows, 2, 64, split_stride=rows * 66, row_stride=66)
    la.sync()
    want = orc.verify(Q, K, V, ctx, window=window)
    assert rel_err(out.float().cpu().numpy().reshape(want.shape), want) < TOL_PAIR


def test_heads_shards(la, orc, synth, cuda):
    import torch

    ctx, m = 6000, 16
    Q, K, V = full_case(synth, 60, ctx, m)
    outs = []
    for r in range(2):
        h0, h1 = head_range(2, r, 8)
        q0, q1 = query_head_range(2, r, 8, 32)
        cache = la.LayerCache(la.MODE_F16, h1 - h0, 64, ctx + m + 64, device=cuda)
        cache.append(dev(K[:, h0:h1], cuda), dev(V[:, h0:h1], cuda), 0)
        outs.append(cache.verify(dev(Q[:, q0:q1], cuda), ctx))
    la.sync()
    got = torch.cat(outs, dim=1).float().cpu().numpy()
    assert rel_err(got, orc.verify(Q, K, V, ctx)) < TOL_PAIR
