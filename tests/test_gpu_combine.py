"""lfm3a_combine against the oracle's merge (dspark.hip:2134-2185) for split counts that take each kernel: up to
64 splits the (row, dim) kernel, beyond the row-per-block kernel; partials from empty splits (max -inf, sum 0)
included, with and without the gate. Tolerance: half an fp16 ulp of the reference plus
3e-4 of the RMS (fp32 summation order and exp2 rounding over up to 400 weights)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("splits", [1, 37, 64, 65, 100, 130, 296, 400])
@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("d", [64, 128])
def test_combine_split_counts(la, orc, synth, cuda, splits, gated, d):
    import torch

    rows = 64
    rng = np.random.default_rng(splits)
    parts = np.empty((splits, rows, d + 2), dtype=np.float32)
    parts[:, :, :d] = rng.normal(size=(splits, rows, d)).astype(np.float32) * 5.0
    parts[:, :, d] = rng.normal(size=(splits, rows)).astype(np.float32) * 3.0
    parts[:, :, d + 1] = rng.uniform(0.5, 40.0, size=(splits, rows)).astype(np.float32)
    empty = rng.random((splits, rows)) < 0.1
    empty[0, 0] = splits > 1   # row 0 keeps a live split
    parts[empty, :d] = 0.0
    parts[empty, d] = -np.inf
    parts[empty, d + 1] = 0.0
    gate = synth.Stream(splits).normal_f16((rows,)) if gated else None
    want = orc.combine(parts, d, gate=gate)
    got = la.combine(torch.from_numpy(parts).to(cuda), rows, splits, d, split_stride=rows * (d + 2), row_stride=d + 2,
                     gate=None if gate is None else torch.from_numpy(gate).to(cuda))
    la.sync()
    got = got.float().cpu().numpy().astype(np.float64)
    want = want.astype(np.float64)
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    assert float(np.max(np.abs(got - want) - half_ulp)) <= 3e-4 * rms


@pytest.mark.parametrize("splits", [40, 100])
def test_verify_partial_many_splits(la, orc, synth, cuda, splits):
    """A shard's merged partial (lfm3a_verify_partial) through either combine kernel: up to 64 splits the
    (row, dim) kernel, beyond the row-per-block kernel; the partial's normalised output against the oracle's
    partial of the same keys."""
    ctx, m = 30000, 16
    case = synth.verify_case(700 + splits, ctx, m)
    K = np.concatenate([case["K"], case["newK"]])
    V = np.concatenate([case["V"], case["newV"]])
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx + m + 64, device=cuda)
    cache.append(torch_dev(K, cuda), torch_dev(V, cuda), 0)
    b, e = 10048, ctx + m
    got = cache.verify_partial(torch_dev(case["Q"], cuda), b, e, ctx, splits=splits)
    la.sync()
    got = got.cpu().numpy()
    want = orc.verify_partial(case["Q"], K, V, b, e, ctx)
    go = got[:, :64] / got[:, 65:66]
    wo = want[:, :64] / want[:, 65:66]
    assert np.max(np.abs(go - wo)) / np.sqrt(np.mean(wo ** 2)) < 4e-3


def torch_dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
