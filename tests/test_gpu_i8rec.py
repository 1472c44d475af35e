"""The reference's own attention arithmetic on its own cache bytes (MODE_I8REC 264-byte records):

* lfm3a_quantize_q (kernels/prefill_attn.hip:120-135) bit-exact against the oracle's restatement, at head_dim 128
  and 64, with zero, tiny and large rows and a strided q;
* lfm3a_verify_attention_i8 (kernels/dspark.hip:1824-2185: int8 Q x int8 K per 32-dim group, P = fp16(p vs 4096)
  x int8 V) against the oracle's restatement of the same arithmetic (4e-3 of the output RMS beyond half an fp16
  ulp: the exponentials and the fp32 summation order differ, and each side rounds P to fp16 against its own
  running maxima) and against exact fp64 attention over the same int8 values (the records' K and V, the
  quantised Q) within 2e-3, at the reference model's 16/4/128 geometry (m = 1..16, windows, short contexts) and
  the benchmark's 32/8/64 one. The records come from the library's own append (bit-exact against the oracle's
  records, checked here too)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_PAIR = 4e-3


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


@pytest.mark.parametrize("d", [128, 64])
def test_quantize_q_bit_exact(la, orc, synth, cuda, d):
    import torch

    t, qh = 37, 16
    q = synth.Stream(800 + d).normal_f16((t, qh, d))
    q[0, 0] = 0                                   # amax 0: scale 1e-20
    q[1, 1] = np.float16(3e-5) * q[1, 1]          # tiny values (subnormal fp16 included)
    q[2, 2] = np.float16(60000.0)                 # large
    q[3, :, :7] = np.float16(-2.5)                # ties of x / scale
    got = la.quantize_q(dev(q, cuda))
    la.sync()
    want = orc.quantize_q(q)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want)
    # a strided view of raw projections: rows of 3 * qh * d halves, the queries first
    raw = synth.Stream(801 + d).normal_f16((t, 3 * qh * d))
    qd = dev(raw, cuda)
    got = la.quantize_q(qd, q_heads=qh, head_dim=d)
    la.sync()
    want = orc.quantize_q(np.ascontiguousarray(raw[:, :qh * d]).reshape(t, qh, d))
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want)
    del torch


def f64_attention(qbuf, rec, m, q_heads, ctx_len, window=0):
    """Exact attention over the int8 values: the quantised Q, the records' K and V (each times its scale)."""
    Kd, Vd = orc_mod().dequantize_rec(rec)
    d = Kd.shape[2]
    Q = orc_mod().dequantize_q(qbuf, d).reshape(m, q_heads, d)
    g = q_heads // Kd.shape[1]
    out = np.zeros((m, q_heads, d))
    start = max(0, ctx_len - window + 1) if window > 0 else 0
    for t in range(m):
        qpos = ctx_len + t
        lo = max(start, qpos - window + 1) if window > 0 else start
        idx = np.concatenate([np.arange(lo, ctx_len), np.arange(ctx_len, qpos + 1)])
        for qq in range(q_heads):
            h = qq // g
            s = Kd[idx, h] @ Q[t, qq] / np.sqrt(d)
            p = np.exp(s - s.max())
            out[t, qq] = (p / p.sum()) @ Vd[idx, h]
    return out


def orc_mod():
    from oracle import oracle

    return oracle


def run_i8(la, orc, synth, cuda, seed, ctx, m, q_heads, kv_heads, d, window=0, splits=0, theta=1e6, factor=0.5):
    case = synth.verify_case(seed, ctx, m, q_heads=q_heads, kv_heads=kv_heads, head_dim=d)
    K = np.concatenate([case["K"], case["newK"]])
    V = np.concatenate([case["V"], case["newV"]])
    rope_np = la.rope_table(theta, factor, d, ctx + m + 1)
    cache = la.LayerCache(la.MODE_I8REC, kv_heads, d, ctx + m + 64, device=cuda)
    cache.append(dev(K, cuda), dev(V, cuda), 0, rope=dev(rope_np.view(np.float16), cuda))
    qbuf = la.quantize_q(dev(case["Q"], cuda))
    out = cache.verify_i8(qbuf, m, q_heads, ctx, window=window, splits=splits)
    la.sync()
    rec = cache.logical(ctx + m)["rec"]
    want_rec = orc.kv_append_i8rec(K, V, 0, rope=rope_np.view(np.float16))
    assert np.array_equal(rec, want_rec)
    qb = qbuf.cpu().numpy().view(np.uint32)
    got = out.float().cpu().numpy()
    pair = rel_err(got, orc.verify_i8rec(qb, m, q_heads, rec, ctx, window=window, splits=max(splits, 1)))
    exact = rel_err(got, f64_attention(qb, rec, m, q_heads, ctx, window))
    return pair, exact


@pytest.mark.parametrize("ctx,m,window,splits", [(3000, 9, 0, 0), (3000, 8, 0, 7), (131, 1, 0, 0), (5, 16, 0, 0),
                                                  (4000, 3, 256, 0), (20000, 16, 0, 0), (1000, 9, 0, 1)])
def test_verify_i8_reference_geometry(la, orc, synth, cuda, ctx, m, window, splits):
    pair, exact = run_i8(la, orc, synth, cuda, 900 + m + ctx % 97, ctx, m, 16, 4, 128, window, splits)
    assert pair < TOL_PAIR and exact < TOL, (pair, exact)


@pytest.mark.parametrize("ctx,m", [(5000, 8), (777, 1)])
def test_verify_i8_benchmark_geometry(la, orc, synth, cuda, ctx, m):
    pair, exact = run_i8(la, orc, synth, cuda, 950 + m, ctx, m, 32, 8, 64, factor=1.0)
    assert pair < TOL_PAIR and exact < TOL, (pair, exact)


def test_verify_i8_published_case(la, orc, synth, cuda):
    """The reference's published verify measurement (benchmarks/verify_attention.txt: 8 verified tokens at its
    16/4/128 geometry over a long context; worst error 3.80e-4 against fp64) at 32768 cached tokens: the worst
    error against fp64 over the same int8 values, printed beside the bound."""
    pair, exact = run_i8(la, orc, synth, cuda, 960, 32768, 8, 16, 4, 128)
    print(f"mode A verify, 8 tokens over 32768: max error vs fp64 {exact:.2e} of the RMS (beyond half an fp16 ulp); "
          f"vs the oracle {pair:.2e}")
    assert pair < TOL_PAIR and exact < TOL


# ---------------------------------------------------------------- prefill over the records
TOL_PREFILL = 2e-2   # against the oracle's restatement: u8 roundings that flip with the exponentials' last bits


def run_prefill_i8(la, orc, synth, cuda, seed, context, tokens, q_heads, kv_heads, d, window=0, splits=1, exact=False):
    n = context + tokens
    case = synth.prefill_case(seed, n, q_heads=q_heads, kv_heads=kv_heads, head_dim=d)
    rope_np = la.rope_table(1e6, 0.5 if d == 128 else 1.0, d, n + 1)
    cache = la.LayerCache(la.MODE_I8REC, kv_heads, d, n + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0, rope=dev(rope_np.view(np.float16), cuda))
    qbuf = la.quantize_q(dev(case["Q"][context:], cuda))
    out = cache.prefill_i8(qbuf, tokens, q_heads, context, window=window, splits=splits, exact=exact)
    la.sync()
    rec = cache.logical(n)["rec"]
    assert np.array_equal(rec, orc.kv_append_i8rec(case["K"], case["V"], 0, rope=rope_np.view(np.float16)))
    qb = qbuf.cpu().numpy().view(np.uint32)
    got = out.float().cpu().numpy()
    if splits <= 0:
        splits = la.lib().lfm3a_prefill_i8_splits(tokens, q_heads, context, window, 0)
    want = orc.prefill_i8rec(qb, tokens, q_heads, rec, context, window=window, splits=splits, exact=exact)
    return got, want, splits


@pytest.mark.parametrize("context,tokens,window,splits", [(0, 70, 0, 1), (200, 40, 0, 1), (300, 33, 100, 1),
                                                          (3000, 96, 0, 3), (5000, 64, 0, 0), (1000, 32, 256, 1),
                                                          (129, 1, 0, 1)])
def test_prefill_i8_reference_geometry(la, orc, synth, cuda, context, tokens, window, splits):
    """lfm3a_prefill_attention_i8 (prefill_attn.hip:212-505 over the records) against the oracle's restatement with
    the same 32-token blocks and key splits: within 2e-2 of the RMS beyond half an fp16 ulp, and within 1e-3 on
    average. The default split count of a short chunk over a long context is above 1."""
    got, want, used = run_prefill_i8(la, orc, synth, cuda, 1000 + tokens + context, context, tokens, 16, 4, 128,
                                     window, splits)
    if splits == 0:
        assert used > 1
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    assert rel_err(got, want) < TOL_PREFILL
    assert float(np.mean(np.abs(got - want))) / rms < 1e-3


def test_prefill_i8_benchmark_geometry(la, orc, synth, cuda):
    got, want, _ = run_prefill_i8(la, orc, synth, cuda, 1100, 150, 40, 32, 8, 64)
    assert rel_err(got, want) < TOL_PREFILL


@pytest.mark.parametrize("context,tokens,window,splits", [(0, 70, 0, 1), (300, 33, 100, 1), (3000, 96, 0, 3),
                                                          (5000, 64, 0, 0), (129, 1, 0, 1)])
def test_prefill_i8_exact_reference_geometry(la, orc, synth, cuda, context, tokens, window, splits):
    """The exact variant over the records (prefill_attn_exact.hip:173-344: exact running max, fp16 P' = p v_scale
    4096 x V) against the oracle's restatement with the same blocks and splits, within the two-rounding bar of the
    fp16 probabilities (4e-3 of the RMS beyond half an fp16 ulp); the oracle itself is held to exact fp64 attention
    over the same int8 values in test_oracle_math.py."""
    got, want, _ = run_prefill_i8(la, orc, synth, cuda, 1200 + tokens + context, context, tokens, 16, 4, 128,
                                  window, splits, exact=True)
    assert rel_err(got, want) < TOL_PAIR


def test_prefill_i8_exact_benchmark_geometry(la, orc, synth, cuda):
    got, want, _ = run_prefill_i8(la, orc, synth, cuda, 1300, 150, 40, 32, 8, 64, exact=True)
    assert rel_err(got, want) < TOL_PAIR
