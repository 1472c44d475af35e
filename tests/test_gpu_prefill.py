"""Prefill attention on the GPU (tcgen05) against the oracle and exact fp64 attention.

Errors are measured beyond half an fp16 ulp of the reference (the fp16 output's own rounding) and relative
to the reference RMS:
  exact (fp16 probabilities, fp16 V):  <= 4e-3 against fp64 and against the oracle. Rows with a handful
      of keys carry the fp16 rounding of single probabilities (2^-11 each) almost undiluted.
  int8-PV (u8 probabilities per row and 64-key tile, int8 V per 64-token block): <= 2e-2 against the oracle
      of the same arithmetic, whose int8 V is bit-identical to the cache's.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_EXACT = 4e-3
TOL_I8 = 2e-2


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want, rows=None):
    want = want.astype(np.float64)
    got = got.astype(np.float64)
    if rows is not None:
        want, got = want[rows], got[rows]
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got - want) - half_ulp, 0.0, None))) / rms


def run(la, synth, cuda, seed, context, T, window, exact):
    case = synth.prefill_case(seed, context + T)
    cache = la.LayerCache(la.MODE_F16, 8, 64, context + T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    out = cache.prefill(dev(case["Q"][context:], cuda), context, window=window, exact=exact)
    la.sync()
    return case, cache, out.float().cpu().numpy()


CASES = [(0, 32, 0), (0, 64, 0), (0, 100, 0), (37, 100, 0), (160, 300, 100), (0, 640, 0), (1000, 96, 256)]


@pytest.mark.parametrize("context,T,window", CASES)
def test_prefill_exact(la, orc, synth, cuda, context, T, window):
    case, _, got = run(la, synth, cuda, 60 + T, context, T, window, True)
    n = context + T
    q = case["Q"][context:]
    want = orc.attention_f64(q, context, case["K"], case["V"], n, window=window)
    assert rel_err(got, want) < TOL_EXACT
    emu = orc.prefill_exact(q, context, case["K"], case["V"], window=window)
    assert rel_err(got, emu) < TOL_EXACT


@pytest.mark.parametrize("context,T,window", CASES)
def test_prefill_i8pv(la, orc, synth, cuda, context, T, window):
    case, cache, got = run(la, synth, cuda, 70 + T, context, T, window, False)
    n = context + T
    q = case["Q"][context:]
    logical = cache.logical(n)
    v8, vs = orc.quantize_v8(case["V"], n)
    assert np.array_equal(logical["V8"], v8)
    emu = orc.prefill_i8pv(q, context, case["K"], v8, vs, window=window)
    assert rel_err(got, emu) < TOL_I8


def test_prefill_c4_sampled_rows(la, orc, synth, cuda):
    """Config 4 at full size (T = 32768 causal, seed 3), both variants, checked on every 257th query row."""
    import torch

    T = 32768
    case = synth.prefill_case(3, T)
    cache = la.LayerCache(la.MODE_F16, 8, 64, T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    q = dev(case["Q"], cuda)
    ex = cache.prefill(q, 0, exact=True)
    i8 = cache.prefill(q, 0, exact=False)
    la.sync()
    rows = np.arange(0, T, 257)
    want = orc.attention_f64(case["Q"], 0, case["K"], case["V"], T, row_step=257)
    assert rel_err(ex.float().cpu().numpy(), want, rows) < TOL_EXACT
    v8, vs = orc.quantize_v8(case["V"], T)
    emu = orc.prefill_i8pv(case["Q"], 0, case["K"], v8, vs, row_step=257)
    assert rel_err(i8.float().cpu().numpy(), emu, rows) < TOL_I8
    assert torch.isfinite(ex).all() and torch.isfinite(i8).all()


SPLIT_CASES = [(20000, 64, 0), (5000, 100, 2000), (3000, 32, 0), (1000, 200, 0)]


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("context,T,window", SPLIT_CASES)
def test_prefill_key_splits(la, orc, synth, cuda, context, T, window, exact):
    """A short chunk over a long context is split along the keys (lfm3a_prefill_splits) and merged; checked
    against the oracle with the same split and, for exact, against fp64 attention."""
    splits = la.lib().lfm3a_prefill_splits(T, 32, context, window, 0)
    assert splits > 1
    case, cache, got = run(la, synth, cuda, 80 + T, context, T, window, exact)
    n = context + T
    q = case["Q"][context:]
    if exact:
        emu = orc.prefill_exact(q, context, case["K"], case["V"], window=window, splits=splits)
        assert rel_err(got, emu) < TOL_EXACT
        assert rel_err(got, orc.attention_f64(q, context, case["K"], case["V"], n, window=window)) < TOL_EXACT
    else:
        v8, vs = orc.quantize_v8(case["V"], n)
        emu = orc.prefill_i8pv(q, context, case["K"], v8, vs, window=window, splits=splits)
        assert rel_err(got, emu) < TOL_I8


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("context,T", [(37, 100), (3000, 64)])
def test_prefill_fused_glue(la, orc, synth, cuda, context, T, exact):
    """lfm3a_prefill_attention_fused: raw row-strided query projections, normalised and rotated in the
    kernel, give bit for bit the plain call on the oracle's q_norm_rope output; the fused output gate equals
    gate_mul of that output, up to one fp16 ulp where the device's and the host's expf round the sigmoid
    differently. (3000, 64) runs split along the keys, where the gate is applied after the combine."""
    case = synth.prefill_case(90 + T, context + T)
    cache = la.LayerCache(la.MODE_F16, 8, 64, context + T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    s = synth.Stream(95)
    width = 32 * 64 + 3 * 64   # a projection row: the 32 query heads, then other columns
    f = s.normal_f16((T, width))
    qnorm = (1.0 + 0.25 * s.normal_f16((64,)).astype(np.float32)).astype(np.float16)
    table = orc.rope_table(1e6, 1.0, 64, context + T + 1)
    gate = s.normal_f16((T, 40))
    fd, qn_d, rope_d = dev(f, cuda), dev(qnorm, cuda), dev(table.view(np.float16), cuda)
    fused = cache.prefill(fd[:, :32 * 64], context, exact=exact, q_norm=qn_d, rope=rope_d, q_heads=32)
    gated = cache.prefill(fd[:, :32 * 64], context, exact=exact, q_norm=qn_d, rope=rope_d, gate=dev(gate, cuda),
                          q_heads=32)
    q_ref = orc.q_norm_rope(f, 32, 64, context, qnorm=qnorm, rope=table)
    plain = cache.prefill(dev(q_ref, cuda), context, exact=exact)
    la.sync()
    plain_np = plain.cpu().numpy()
    assert np.array_equal(fused.cpu().numpy().view(np.uint16), plain_np.view(np.uint16))
    want = orc.gate_mul(plain_np, gate)
    got = gated.cpu().numpy()
    ulps = np.abs(got.view(np.int16).astype(np.int32) - want.view(np.int16).astype(np.int32))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("context,T", [(37, 100), (20000, 64)])
def test_prefill_fused_glue_head_dim_128(la, orc, synth, cuda, context, T, exact):
    """The fused glue at the reference model's geometry (16/4/128, RoPE over half the dims): q_norm_rope with the
    reference's own sum-of-squares order (its wave_sum over the pairs d, d + 64) inside the kernel's Q load gives
    bit for bit the plain call on the oracle's q_norm_rope output; the gate as at head_dim 64. (20000, 64) runs
    split along the keys, the gate applied after the combine."""
    case = synth.prefill_case(190 + T, context + T, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, context + T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    s = synth.Stream(195)
    width = 16 * 128 + 2 * 128 + 48   # a projection row: the 16 query heads, then other columns
    f = s.normal_f16((T, width))
    qnorm = (1.0 + 0.25 * s.normal_f16((128,)).astype(np.float32)).astype(np.float16)
    table = orc.rope_table(1e6, 0.5, 128, context + T + 1)
    gate = s.normal_f16((T, 24))
    fd, qn_d, rope_d = dev(f, cuda), dev(qnorm, cuda), dev(table.view(np.float16), cuda)
    fused = cache.prefill(fd[:, :16 * 128], context, exact=exact, q_norm=qn_d, rope=rope_d, q_heads=16)
    gated = cache.prefill(fd[:, :16 * 128], context, exact=exact, q_norm=qn_d, rope=rope_d, gate=dev(gate, cuda),
                          q_heads=16)
    q_ref = orc.q_norm_rope(f, 16, 128, context, qnorm=qnorm, rope=table)
    plain = cache.prefill(dev(q_ref, cuda), context, exact=exact)
    la.sync()
    plain_np = plain.cpu().numpy()
    assert np.array_equal(fused.cpu().numpy().view(np.uint16), plain_np.view(np.uint16))
    want = orc.gate_mul(plain_np, gate)
    got = gated.cpu().numpy()
    ulps = np.abs(got.view(np.int16).astype(np.int32) - want.view(np.int16).astype(np.int32))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3


# ---------------------------------------------------------------- the reference model's geometry
# 16 query heads, 4 kv heads, head_dim 128 (internal/model/engine.go:22-40). The exact kernel runs two CTAs per
# SM there, as at head_dim 64; the int8-PV kernel one, so its key splits follow lfm3a_prefill_splits with half the
# SM count.
def run_ref(la, synth, cuda, seed, context, T, window, exact):
    case = synth.prefill_case(seed, context + T, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, context + T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    out = cache.prefill(dev(case["Q"][context:], cuda), context, window=window, exact=exact)
    la.sync()
    return case, cache, out.float().cpu().numpy()


REF_CASES = [(0, 32, 0), (0, 100, 0), (37, 100, 0), (160, 300, 100), (1000, 96, 256)]


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("context,T,window", REF_CASES)
def test_prefill_head_dim_128(la, orc, synth, cuda, context, T, window, exact):
    case, cache, got = run_ref(la, synth, cuda, 100 + T + context, context, T, window, exact)
    n = context + T
    q = case["Q"][context:]
    if exact:
        assert rel_err(got, orc.attention_f64(q, context, case["K"], case["V"], n, window=window)) < TOL_EXACT
        assert rel_err(got, orc.prefill_exact(q, context, case["K"], case["V"], window=window)) < TOL_EXACT
    else:
        logical = cache.logical(n)
        v8, vs = orc.quantize_v8(case["V"], n)
        assert np.array_equal(logical["V8"], v8)
        assert rel_err(got, orc.prefill_i8pv(q, context, case["K"], v8, vs, window=window)) < TOL_I8


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("context,T", [(20000, 64), (3000, 32)])
def test_prefill_head_dim_128_key_splits(la, orc, synth, cuda, context, T, exact):
    import torch

    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    splits = la.lib().lfm3a_prefill_splits(T, 16, context, 0, sms if exact else sms // 2)
    assert splits > 1
    case, _, got = run_ref(la, synth, cuda, 110 + T, context, T, 0, exact)
    q = case["Q"][context:]
    if exact:
        assert rel_err(got, orc.prefill_exact(q, context, case["K"], case["V"], splits=splits)) < TOL_EXACT
        assert rel_err(got, orc.attention_f64(q, context, case["K"], case["V"], context + T)) < TOL_EXACT
    else:
        v8, vs = orc.quantize_v8(case["V"], context + T)
        assert rel_err(got, orc.prefill_i8pv(q, context, case["K"], v8, vs, splits=splits)) < TOL_I8


def test_prefill_head_dim_128_sampled_rows(la, orc, synth, cuda):
    """A 2048-token causal prompt at head_dim 128, both variants, on every 37th query row."""
    T = 2048
    case = synth.prefill_case(120, T, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, T + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    q = dev(case["Q"], cuda)
    ex = cache.prefill(q, 0, exact=True)
    i8 = cache.prefill(q, 0, exact=False)
    la.sync()
    rows = np.arange(0, T, 37)
    want = orc.attention_f64(case["Q"], 0, case["K"], case["V"], T, row_step=37)
    assert rel_err(ex.float().cpu().numpy(), want, rows) < TOL_EXACT
    v8, vs = orc.quantize_v8(case["V"], T)
    emu = orc.prefill_i8pv(case["Q"], 0, case["K"], v8, vs, row_step=37)
    assert rel_err(i8.float().cpu().numpy(), emu, rows) < TOL_I8


def test_prefill_head_dim_128_gate_only(la, orc, synth, cuda):
    """The gate alone at head_dim 128 (a plain Q): gate_mul of the plain call's output, within one fp16 ulp where
    the device's and the host's expf round the sigmoid differently."""
    case = synth.prefill_case(121, 64, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, 128, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    gate = synth.Stream(122).normal_f16((64, 16))
    gated = cache.prefill(dev(case["Q"], cuda), 0, exact=True, gate=dev(gate, cuda))
    plain = cache.prefill(dev(case["Q"], cuda), 0, exact=True)
    la.sync()
    want = orc.gate_mul(plain.cpu().numpy(), gate)
    got = gated.cpu().numpy()
    ulps = np.abs(got.view(np.int16).astype(np.int32) - want.view(np.int16).astype(np.int32))
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3
