"""The oracle's restated attention arithmetic against exact fp64 attention, at sizes it finishes in seconds."""
import numpy as np
import pytest


def rel_err(got, want):
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    return float(np.max(np.abs(got.astype(np.float64) - want))) / rms


def build_cache(orc, case, ctx_len, m, theta=1e6):
    table = orc.rope_table(theta, 1.0, 64, ctx_len + m)
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], ctx_len, rope=table)
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    return K, V


@pytest.mark.parametrize("splits", [1, 3, 16])
def test_verify_c1_matches_fp64(orc, synth, splits):
    case = synth.verify_case(0, 1024, 8)
    K, V = build_cache(orc, case, 1024, 8)
    got = orc.verify(case["Q"], K, V, 1024, splits=splits)
    want = orc.attention_f64(case["Q"], 1024, K, V, 1032)
    assert rel_err(got, want) < 2e-3


def test_verify_window_and_gate(orc, synth):
    case = synth.verify_case(5, 700, 5)
    K, V = build_cache(orc, case, 700, 5)
    gate = synth.Stream(9).normal_f16((5, 32))
    got = orc.verify(case["Q"], K, V, 700, window=256, gate=gate, splits=4)
    want = orc.attention_f64(case["Q"], 700, K, V, 705, window=256)
    sig = 1.0 / (1.0 + np.exp(-gate.astype(np.float64)))
    assert rel_err(got, want * sig[..., None]) < 2e-3


def test_verify_split_invariance(orc, synth):
    case = synth.verify_case(1, 3000, 16)
    K, V = build_cache(orc, case, 3000, 16)
    a = orc.verify(case["Q"], K, V, 3000, splits=1)
    b = orc.verify(case["Q"], K, V, 3000, splits=37)
    assert rel_err(b, a) < 1e-3


@pytest.mark.parametrize("context,window", [(0, 0), (96, 0), (160, 100)])
def test_prefill_exact_and_i8_match_fp64(orc, synth, context, window):
    t = 200
    case = synth.prefill_case(3, context + t)
    K, V, Q = case["K"], case["V"], case["Q"][context:]
    V8, vs = orc.quantize_v8(V, context + t)
    want = orc.attention_f64(Q, context, K, V, context + t, window=window)
    ex = orc.prefill_exact(Q, context, K, V, window=window)
    # fp16 probabilities carry a 2^-11 relative rounding each: a few 1e-3 of the output RMS against fp64.
    assert rel_err(ex, want) < 4e-3
    # The int8 arithmetic is checked against fp64 attention over the dequantised int8 V: what remains is
    # the u8 rounding of the probabilities (per row and 64-key tile), up to ~8% of the output RMS at
    # worst and far less on average. The 2e-2 bar applies between implementations of the same arithmetic.
    i8 = orc.prefill_i8pv(Q, context, K, V8, vs, window=window)
    n = context + t
    v_dq = (V8[:n].astype(np.float32) * np.repeat(vs, 64, axis=0)[:n, :, None]).astype(np.float16)
    want_dq = orc.attention_f64(Q, context, K, v_dq, n, window=window)
    rms = float(np.sqrt(np.mean(want_dq.astype(np.float64) ** 2)))
    assert rel_err(i8, want_dq) < 0.15
    assert float(np.mean(np.abs(i8 - want_dq))) / rms < 5e-3


def test_prefill_row_sampling(orc, synth):
    case = synth.prefill_case(4, 300)
    full = orc.prefill_exact(case["Q"], 0, case["K"], case["V"])
    some = orc.prefill_exact(case["Q"], 0, case["K"], case["V"], row_step=7)
    assert np.array_equal(full[::7], some[::7])
    assert not some[1].any()


def test_prefill_split_merge(orc, synth):
    """The oracle's key-split prefill (per-split running maxima, log-sum-exp merge) against its unsplit pass
    and exact fp64 attention."""
    ctx, T = 3000, 40
    case = synth.prefill_case(90, ctx + T)
    q = case["Q"][ctx:]
    want = orc.attention_f64(q, ctx, case["K"], case["V"], ctx + T).astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    for splits in (1, 3, 6):
        got = orc.prefill_exact(q, ctx, case["K"], case["V"], splits=splits)
        assert float(np.max(np.abs(got - want))) / rms < 2e-3


def records_case(orc, synth, seed, n, q_heads, kv_heads, d, theta=1e6, factor=0.5):
    """Int8 records of n positions (the oracle's append with RoPE) and the quantised queries of the last tokens."""
    case = synth.prefill_case(seed, n, q_heads=q_heads, kv_heads=kv_heads, head_dim=d)
    rope = orc.rope_table(theta, factor, d, n + 1).view(np.float16)
    rec = orc.kv_append_i8rec(case["K"], case["V"], 0, rope=rope)
    return case, rec


def f64_prefill_over_records(orc, qbuf, rec, tokens, q_heads, context, window=0):
    """Exact causal attention over the int8 values: the records' K and V times their scales, the quantised Q."""
    Kd, Vd = orc.dequantize_rec(rec)
    d = Kd.shape[2]
    Q = orc.dequantize_q(qbuf, d).reshape(tokens, q_heads, d)
    g = q_heads // Kd.shape[1]
    out = np.zeros((tokens, q_heads, d))
    for t in range(tokens):
        qpos = context + t
        lo = max(0, qpos - window + 1) if window > 0 else 0
        for qh in range(q_heads):
            s = Kd[lo:qpos + 1, qh // g] @ Q[t, qh] / np.sqrt(d)
            p = np.exp(s - s.max())
            out[t, qh] = (p / p.sum()) @ Vd[lo:qpos + 1, qh // g]
    return out


@pytest.mark.parametrize("d,context,tokens,window", [(128, 200, 40, 0), (128, 0, 70, 0), (128, 300, 33, 100),
                                                     (64, 150, 40, 0)])
def test_prefill_i8rec_matches_fp64(orc, synth, d, context, tokens, window):
    """The restated prefill over the reference's records (prefill_attn.hip:212-505: lazy max, u8 P' per row and
    64-key tile) against exact attention over the same int8 values: what remains is the u8 rounding of the
    probabilities, up to ~8% of the output RMS at worst and far less on average (the bars of the int8-PV
    restatement); and the same result within 1e-2 whatever the key splits (the u8 rounding is per tile, and the
    splits only move the running maxima)."""
    qh, kvh = (16, 4) if d == 128 else (32, 8)
    case, rec = records_case(orc, synth, 500 + tokens + context, context + tokens, qh, kvh, d)
    qbuf = orc.quantize_q(case["Q"][context:])
    got = orc.prefill_i8rec(qbuf, tokens, qh, rec, context, window=window)
    want = f64_prefill_over_records(orc, qbuf, rec, tokens, qh, context, window)
    rms = float(np.sqrt(np.mean(want ** 2)))
    assert rel_err(got, want) < 0.15
    assert float(np.mean(np.abs(got - want))) / rms < 5e-3
    split = orc.prefill_i8rec(qbuf, tokens, qh, rec, context, window=window, splits=3)
    assert rel_err(split, got) < 1e-2


@pytest.mark.parametrize("d,context,tokens,window", [(128, 200, 40, 0), (128, 300, 33, 100), (64, 150, 40, 0)])
def test_prefill_i8rec_exact_matches_fp64(orc, synth, d, context, tokens, window):
    """The restated exact prefill over the records (prefill_attn_exact.hip:173-344: exact running max, fp16
    P' = p * v_scale * 4096) against exact attention over the same int8 values: within 4e-3 of the RMS (the fp16
    probabilities), and the same within 3e-3 whatever the key splits (each split rounds its P' to fp16 against
    its own running maximum)."""
    qh, kvh = (16, 4) if d == 128 else (32, 8)
    case, rec = records_case(orc, synth, 600 + tokens + context, context + tokens, qh, kvh, d)
    qbuf = orc.quantize_q(case["Q"][context:])
    got = orc.prefill_i8rec(qbuf, tokens, qh, rec, context, window=window, exact=True)
    want = f64_prefill_over_records(orc, qbuf, rec, tokens, qh, context, window)
    assert rel_err(got, want) < 4e-3
    split = orc.prefill_i8rec(qbuf, tokens, qh, rec, context, window=window, splits=3, exact=True)
    assert rel_err(split, got) < 3e-3
