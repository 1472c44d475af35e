"""lfm3a_verify_attention_static (split partials in the library's fixed device scratch) against
lfm3a_verify_attention (caller's workspace), both called through the C ABI, and against exact fp64 attention.

Two static calls in a row on one stream share the one scratch array: a 16-token verify over 32768 cached
tokens (M = 64 kernel, 37 splits) and then a 24-token verify over 5000 with a window (M = 128 kernel). Each
output must match the workspace entry point within the verify tolerance between implementations (4e-3 of the
output RMS beyond half an fp16 ulp) and exact fp64 attention within the verify tolerance (2e-3). A call whose partials exceed the scratch
must fail with LFM3A_EWORKSPACE before launching anything. The file sorts last so that it also runs after every
other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_PAIR = 4e-3
TOL_F64 = 2e-3


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


def make_cache(la, synth, cuda, seed, ctx_len, m):
    case = synth.verify_case(seed, ctx_len, m)
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx_len + m + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    cache.append(dev(case["newK"], cuda), dev(case["newV"], cuda), ctx_len)
    return case, cache


def call_static(la, cache, q, ctx_len, window, out, splits, stream):
    m, qh = q.shape[0], q.shape[1]
    return la.lib().lfm3a_verify_attention_static(ctypes.byref(cache.view), q.data_ptr(), m, qh, ctx_len, window,
                                                  None, out.data_ptr(), splits, stream)


def test_static_scratch_matches_workspace_entry(la, orc, synth, cuda):
    import torch

    stream = torch.cuda.current_stream(cuda).cuda_stream
    runs = [(31, 32768, 16, 0), (32, 5000, 24, 777)]
    cases = [make_cache(la, synth, cuda, seed, ctx, m) for seed, ctx, m, _ in runs]
    qs = [dev(case["Q"], cuda) for case, _ in cases]
    outs = [torch.empty_like(q) for q in qs]
    for (seed, ctx, m, window), (case, cache), q, out in zip(runs, cases, qs, outs):
        assert la.verify_splits(cache.layout, ctx, m, window) > 1
        assert call_static(la, cache, q, ctx, window, out, 0, stream) == la.OK, la.lib().lfm3a_last_error()
    la.sync()
    for (seed, ctx, m, window), (case, cache), q, out in zip(runs, cases, qs, outs):
        want = cache.verify(q, ctx, window=window)
        la.sync()
        got = out.float().cpu().numpy()
        assert rel_err(got, want.float().cpu().numpy()) < TOL_PAIR
        K = np.concatenate([case["K"], case["newK"]])
        V = np.concatenate([case["V"], case["newV"]])
        assert rel_err(got, orc.attention_f64(case["Q"], ctx, K, V, ctx + m, window=window)) < TOL_F64


def test_static_scratch_rejects_oversize(la, synth, cuda):
    import torch

    case, cache = make_cache(la, synth, cuda, 33, 32768, 32)
    q = dev(case["Q"], cuda)
    out = torch.zeros_like(q)
    # 32 tokens x 32 query heads x 300 splits x 66 floats = 81 MB > the 16 MiB scratch.
    rc = call_static(la, cache, q, 32768, 0, out, 300, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == la.EWORKSPACE
    assert b"static scratch" in la.lib().lfm3a_last_error()
    la.sync()
    assert not out.any()
