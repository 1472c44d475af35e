"""DSpark verify attention on the GPU against the oracle (same arithmetic) and exact fp64 attention.

Tolerance: max(|gpu - fp64| - ulp16(fp64) / 2) <= 2e-3 x RMS(fp64). The output is fp16, and its own
rounding (half an fp16 ulp, up to ~2e-3 of the RMS for short contexts) is exempt; the arithmetic before it
(fp16 probabilities, fp32 accumulation) must stay within 2e-3. Both the kernel and the oracle round each
probability to fp16 against a running maximum, and those maxima differ with the split/page order, so gpu vs
oracle carries two independent fp16 roundings: that comparison uses 4e-3."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_PAIR = 4e-3


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    """Max error relative to the RMS of want, beyond half an fp16 ulp of want (the output rounding)."""
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


def setup(la, orc, synth, cuda, seed, ctx_len, m, window=0, theta=1e6):
    case = synth.verify_case(seed, ctx_len, m)
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx_len + m + 64, device=cuda)
    rope_np = la.rope_table(theta, 1.0, 64, ctx_len + m + 1)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    cache.append(dev(case["newK"], cuda), dev(case["newV"], cuda), ctx_len, rope=dev(rope_np.view(np.float16), cuda))
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], ctx_len, rope=rope_np.view(np.float16))
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    return case, cache, K, V


@pytest.mark.parametrize("splits", [1, 0, 7])
def test_verify_c1(la, orc, synth, cuda, splits):
    case, cache, K, V = setup(la, orc, synth, cuda, 0, 1024, 8)
    out = cache.verify(dev(case["Q"], cuda), 1024, splits=splits)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.verify(case["Q"], K, V, 1024, splits=max(splits, 1))) < TOL_PAIR
    assert rel_err(got, orc.attention_f64(case["Q"], 1024, K, V, 1032)) < TOL


@pytest.mark.parametrize("m", [1, 3, 9, 16, 17, 32])
def test_verify_token_counts(la, orc, synth, cuda, m):
    case, cache, K, V = setup(la, orc, synth, cuda, 20 + m, 2000, m)
    out = cache.verify(dev(case["Q"], cuda), 2000)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.attention_f64(case["Q"], 2000, K, V, 2000 + m)) < TOL


def test_verify_window_gate(la, orc, synth, cuda):
    case, cache, K, V = setup(la, orc, synth, cuda, 30, 5000, 16)
    gate = synth.Stream(31).normal_f16((16, 32))
    out = cache.verify(dev(case["Q"], cuda), 5000, window=256, gate=dev(gate, cuda))
    la.sync()
    got = out.float().cpu().numpy()
    want = orc.attention_f64(case["Q"], 5000, K, V, 5016, window=256)
    sig = 1.0 / (1.0 + np.exp(-gate.astype(np.float64)))
    assert rel_err(got, want * sig[..., None]) < TOL


@pytest.mark.parametrize("ctx_len", [0, 5, 31, 32, 33, 100])
def test_verify_short_contexts(la, orc, synth, cuda, ctx_len):
    case, cache, K, V = setup(la, orc, synth, cuda, 40 + ctx_len, ctx_len, 16)
    out = cache.verify(dev(case["Q"], cuda), ctx_len)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.attention_f64(case["Q"], ctx_len, K, V, ctx_len + 16)) < TOL


def test_verify_c2_full_size(la, orc, synth, cuda):
    """Config 2 at full size: 32768 cached tokens, 16 drafts (seed 1)."""
    case, cache, K, V = setup(la, orc, synth, cuda, 1, 32768, 16)
    out = cache.verify(dev(case["Q"], cuda), 32768)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.attention_f64(case["Q"], 32768, K, V, 32784)) < TOL


def test_verify_lifecycle_small(la, orc, synth, cuda):
    """Append 16 drafts, verify, keep n and roll back the rest, 12 times; the cache matches the oracle's."""
    s = synth.Stream(50)
    ctx = 700
    k0 = s.normal_f16((ctx, 8, 64))
    v0 = s.normal_f16((ctx, 8, 64))
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx + 16 * 13, device=cuda)
    rope_np = la.rope_table(1e6, 1.0, 64, ctx + 16 * 13)
    rope = dev(rope_np.view(np.float16), cuda)
    cache.append(dev(k0, cuda), dev(v0, cuda), 0)
    K, V = k0.copy(), v0.copy()
    keep = synth.geometric_keep(4, 12)
    for step in range(12):
        nk = s.normal_f16((16, 8, 64))
        nv = s.normal_f16((16, 8, 64))
        q = s.normal_f16((16, 32, 64))
        L = cache.length
        cache.append(dev(nk, cuda), dev(nv, cuda), L, rope=rope)
        out = cache.verify(dev(q, cuda), L)
        ko, vo = orc.kv_append_f16(nk, nv, L, rope=rope_np.view(np.float16))
        Kf, Vf = np.concatenate([K, ko]), np.concatenate([V, vo])
        la.sync()
        assert rel_err(out.float().cpu().numpy(), orc.attention_f64(q, L, Kf, Vf, L + 16)) < TOL
        n = int(keep[step])
        cache.truncate(L + n)
        K, V = Kf[:L + n], Vf[:L + n]
    la.sync()
    got = cache.logical()
    assert got["K"].shape[0] == ctx + int(keep.sum())
    assert np.array_equal(got["K"].view(np.uint16), K.view(np.uint16))
    assert np.array_equal(got["V"].view(np.uint16), V.view(np.uint16))
    v8, sc = orc.quantize_v8(V, V.shape[0])
    assert np.array_equal(got["V8"], v8)
    assert np.array_equal(got["vscale"].view(np.uint32), sc.view(np.uint32))


@pytest.mark.parametrize("ctx,splits", [(20000, 0), (1500, 13)])
def test_verify_dirty_workspace_and_graph_replays(la, orc, synth, cuda, ctx, splits):
    """Nothing in the workspace needs clearing: a workspace full of junk, consecutive calls on it, and replays of
    a captured graph all give the exact-attention result, also with one split per tile (1500 tokens, 13 splits)."""
    import torch

    case, cache, K, V = setup(la, orc, synth, cuda, 90 + splits, ctx, 16)
    want = orc.attention_f64(case["Q"], ctx, K, V, ctx + 16)
    q = dev(case["Q"], cuda)
    sp = splits or la.verify_splits(cache.layout, ctx, 16, 0)
    ws = torch.full((la.lib().lfm3a_verify_workspace_bytes(16, 32, 64, sp),), 0xAB, dtype=torch.uint8, device=cuda)
    outs = [torch.empty_like(q) for _ in range(2)]
    for _ in range(3):
        cache.verify(q, ctx, out=outs[0], workspace=ws, splits=sp)
        la.sync()
        assert rel_err(outs[0].float().cpu().numpy(), want) < TOL
    stream = torch.cuda.Stream(device=cuda)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for o in outs:
            cache.verify(q, ctx, out=o, workspace=ws, splits=sp)
    for _ in range(3):
        for o in outs:
            o.zero_()
        graph.replay()
        torch.cuda.synchronize()
        la.sync()
        for o in outs:
            assert rel_err(o.float().cpu().numpy(), want) < TOL
    del graph


@pytest.mark.parametrize("ctx_len,seed", [(32768, 1), (131072, 2)])
def test_decode_full_size(la, orc, synth, cuda, ctx_len, seed):
    """Decode (m = 1, the scope table's first next row) at the benchmark's context lengths, against fp64."""
    case, cache, K, V = setup(la, orc, synth, cuda, seed, ctx_len, 1)
    out = cache.verify(dev(case["Q"], cuda), ctx_len)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.attention_f64(case["Q"], ctx_len, K, V, ctx_len + 1)) < TOL


@pytest.mark.parametrize("m", [16, 24])
def test_ring_attention(la, orc, synth, cuda, m):
    """The drafter's KV ring (dspark.hip:1070-1412 with RING): 24 ring blocks (768 positions) take a
    1500-token context appended in chunks through the wrapping table (older pages are overwritten), then m
    drafts; the drafts attend the live 600 tokens [ctx_len - 600, ctx_len) and all m drafts, not causally.
    Checked against exact fp64 attention over those keys."""
    ring_blocks, ctx_len, live = 24, 1500, 600
    table = la.ring_table(ring_blocks, (ctx_len + m + 31) // 32 + 1)
    cache = la.LayerCache(la.MODE_F16, 8, 64, len(table) * 32, device=cuda, block_table=dev(table, cuda),
                          pool_blocks=ring_blocks)
    case = synth.verify_case(50 + m, ctx_len, m)
    rope_np = orc.rope_table(1e6, 1.0, 64, ctx_len + m + 1)
    rope = dev(rope_np.view(np.float16), cuda)
    for p0 in range(0, ctx_len, 250):
        cache.append(dev(case["K"][p0:p0 + 250], cuda), dev(case["V"][p0:p0 + 250], cuda), p0, rope=rope)
    cache.append(dev(case["newK"], cuda), dev(case["newV"], cuda), ctx_len, rope=rope)
    ctx_lo = ctx_len - live
    out = cache.ring_attention(dev(case["Q"], cuda), ctx_lo, ctx_len)
    la.sync()
    K, V = orc.kv_append_f16(np.concatenate([case["K"], case["newK"]]), np.concatenate([case["V"], case["newV"]]), 0,
                             rope=rope_np)
    kh = np.repeat(K[ctx_lo:].astype(np.float64), 4, axis=1)   # query head 4 h + j reads kv head h
    vh = np.repeat(V[ctx_lo:].astype(np.float64), 4, axis=1)
    s = np.einsum("mhd,nhd->hmn", case["Q"].astype(np.float64), kh) / 8.0
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    want = np.einsum("hmn,nhd->mhd", p, vh)
    assert rel_err(out.float().cpu().numpy(), want) < TOL


@pytest.mark.parametrize("ctx_len,m,splits", [(32768, 16, 0), (1000, 8, 0), (1020, 16, 0), (5, 16, 0),
                                               (2000, 24, 0), (4000, 16, 31)])
def test_verify_round_matches_two_calls(la, orc, synth, cuda, ctx_len, m, splits):
    """lfm3a_verify_round (the drafts' append fused into the attention kernel for m <= 16; 1020 + 16 touches two
    int8 V blocks; m = 24 and 31 splits of 4000 keys take the separate append) leaves the cache bytes of
    lfm3a_kv_append + lfm3a_verify_attention bit for bit, over three rounds with rollbacks between. The output
    matches within the two-rounding tolerance (the appending split holds fewer key tiles, so the splits round
    their fp16 probabilities against different maxima) and exact fp64 attention within 2e-3."""
    case = synth.verify_case(60 + m, ctx_len, m)
    rope_np = la.rope_table(1e6, 1.0, 64, ctx_len + 4 * m + 1)   # rows for every round's drafts
    rope = dev(rope_np.view(np.float16), cuda)
    caches = []
    for _ in range(2):
        c = la.LayerCache(la.MODE_F16, 8, 64, ctx_len + 4 * m + 64, device=cuda)
        c.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
        caches.append(c)
    fused, plain = caches
    s = synth.Stream(61)
    length = ctx_len - 3 if ctx_len > 8 else ctx_len
    fused.truncate(length)
    plain.truncate(length)
    for r in range(3):
        nk, nv = dev(s.normal_f16((m, 8, 64)), cuda), dev(s.normal_f16((m, 8, 64)), cuda)
        q = dev(s.normal_f16((m, 32, 64)), cuda)
        a = fused.verify_round(nk, nv, q, length, rope=rope, splits=splits)
        plain.append(nk, nv, length, rope=rope)
        b = plain.verify(q, length, splits=splits)
        la.sync()
        ao = a.float().cpu().numpy()
        assert rel_err(ao, b.float().cpu().numpy()) < TOL_PAIR
        ga, gb = fused.logical(length + m), plain.logical(length + m)
        for key in ("K", "V", "V8", "vscale", "page_scale"):
            assert np.array_equal(ga[key], gb[key]), key
        K = ga["K"][:length + m].view(np.float16)
        V = ga["V"][:length + m].view(np.float16)
        assert rel_err(ao, orc.attention_f64(q.cpu().numpy(), length, K, V, length + m)) < TOL
        keep = (r * 5 + 3) % m + 1
        length += keep
        fused.truncate(length)
        plain.truncate(length)


@pytest.mark.parametrize("d,ctx_len,timeout_ms", [(64, 3000, 10000), (128, 2000, 10000), (64, 3000, 0), (64, 3000, -1)])
def test_verify_round_host(la, orc, synth, cuda, d, ctx_len, timeout_ms):
    """lfm3a_verify_round_host (the drafts copied in from pinned host memory, the round, the output copied back,
    the stream waited for: bounded, unbounded, or by the caller) gives the bytes of lfm3a_verify_round on the same
    drafts in the host buffer, and the same cache; the output within 2e-3 of exact fp64 attention. Both
    geometries."""
    import torch

    qh, kvh = (32, 8) if d == 64 else (16, 4)
    m = 16 if d == 64 else 9
    case = synth.verify_case(70 + d, ctx_len, m, q_heads=qh, kv_heads=kvh, head_dim=d)
    rope_np = la.rope_table(1e6, 1.0 if d == 64 else 0.5, d, ctx_len + m + 1)
    rope = dev(rope_np.view(np.float16), cuda)
    caches = []
    for _ in range(2):
        c = la.LayerCache(la.MODE_F16, kvh, d, ctx_len + m + 64, device=cuda)
        c.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
        caches.append(c)
    host, plain = caches
    packed = np.concatenate([case["Q"].reshape(-1), case["newK"].reshape(-1), case["newV"].reshape(-1)])
    hin = torch.from_numpy(packed).pin_memory()
    din = torch.empty(hin.shape, dtype=torch.float16, device=cuda)
    hout = torch.zeros((m, qh, d), dtype=torch.float16).pin_memory()
    host.verify_round_host(hin, din, hout, m, qh, ctx_len, rope=rope, timeout_ms=timeout_ms)
    if timeout_ms < 0:
        torch.cuda.current_stream().synchronize()
    got = hout.numpy().copy()   # the stream has finished: the host buffer holds the output
    want = plain.verify_round(dev(case["newK"], cuda), dev(case["newV"], cuda), dev(case["Q"], cuda), ctx_len,
                              rope=rope)
    la.sync()
    assert np.array_equal(got.view(np.uint16), want.cpu().numpy().view(np.uint16))
    ga, gb = host.logical(ctx_len + m), plain.logical(ctx_len + m)
    for key in ("K", "V", "V8", "vscale"):
        assert np.array_equal(ga[key], gb[key]), key
    K = ga["K"][:ctx_len + m].view(np.float16)
    V = ga["V"][:ctx_len + m].view(np.float16)
    assert rel_err(got, orc.attention_f64(case["Q"], ctx_len, K, V, ctx_len + m)) < TOL


# ---------------------------------------------------------------- the reference model's geometry
# LFM3-1.7B itself (internal/model/engine.go:22-40): 16 query heads, 4 kv heads, head_dim 128, RoPE theta 1e6 over
# half the dimensions (factor 0.5, engine.go:333-338). verify_m64_kernel<128> serves up to 16 tokens (the
# reference verifies at most 9: an anchor and 8 drafts, dspark.hip:65).
def setup_ref(la, orc, synth, cuda, seed, ctx_len, m):
    case = synth.verify_case(seed, ctx_len, m, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, ctx_len + m + 64, device=cuda)
    rope_np = la.rope_table(1e6, 0.5, 128, ctx_len + m + 1)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    cache.append(dev(case["newK"], cuda), dev(case["newV"], cuda), ctx_len, rope=dev(rope_np.view(np.float16), cuda))
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], ctx_len, rope=rope_np.view(np.float16))
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    return case, cache, K, V


@pytest.mark.parametrize("ctx_len,m,splits", [(2000, 1, 0), (2000, 9, 0), (2000, 16, 0), (2000, 9, 1), (33, 9, 0),
                                              (0, 16, 0), (32768, 9, 0)])
def test_verify_head_dim_128(la, orc, synth, cuda, ctx_len, m, splits):
    case, cache, K, V = setup_ref(la, orc, synth, cuda, 60 + m + ctx_len % 97, ctx_len, m)
    out = cache.verify(dev(case["Q"], cuda), ctx_len, splits=splits)
    la.sync()
    got = out.float().cpu().numpy()
    assert rel_err(got, orc.attention_f64(case["Q"], ctx_len, K, V, ctx_len + m)) < TOL
    assert rel_err(got, orc.verify(case["Q"], K, V, ctx_len, splits=max(splits, 1))) < TOL_PAIR


def test_verify_head_dim_128_window_gate(la, orc, synth, cuda):
    """A sliding-window layer (window 256, engine.go:36) with the output gate."""
    case, cache, K, V = setup_ref(la, orc, synth, cuda, 70, 5000, 9)
    gate = synth.Stream(71).normal_f16((9, 16))
    out = cache.verify(dev(case["Q"], cuda), 5000, window=256, gate=dev(gate, cuda))
    la.sync()
    want = orc.attention_f64(case["Q"], 5000, K, V, 5009, window=256)
    sig = 1.0 / (1.0 + np.exp(-gate.astype(np.float64)))
    assert rel_err(out.float().cpu().numpy(), want * sig[..., None]) < TOL


def test_verify_head_dim_128_partials(la, orc, synth, cuda):
    """Two sequence shards' (acc, max, sum) partials at head_dim 128, merged by the combine."""
    import torch

    ctx, m = 6000, 9
    case, cache, K, V = setup_ref(la, orc, synth, cuda, 72, ctx, m)
    q = dev(case["Q"], cuda)
    cut = 3072
    parts = [cache.verify_partial(q, 0, cut, ctx), cache.verify_partial(q, cut, ctx + m, ctx)]
    la.sync()
    for part, (b, e) in zip(parts, [(0, cut), (cut, ctx + m)]):
        got = part.cpu().numpy()
        want = orc.verify_partial(case["Q"], K, V, b, e, ctx)
        g = got[:, :128] / got[:, 129:130]
        w = want[:, :128] / want[:, 129:130]
        assert float(np.max(np.abs(g - w))) / float(np.sqrt(np.mean(w.astype(np.float64) ** 2))) < TOL_PAIR
    rows = m * 16
    out = la.combine(torch.stack(parts), rows, 2, 128, split_stride=rows * 130, row_stride=130)
    la.sync()
    want = orc.attention_f64(case["Q"], ctx, K, V, ctx + m)
    assert rel_err(out.float().cpu().numpy().reshape(want.shape), want) < TOL


def test_verify_head_dim_128_rejects_more_than_16_tokens(la, synth, cuda):
    case = synth.verify_case(73, 100, 17, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, 256, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    with pytest.raises(la.LFM3AError) as e:
        cache.verify(dev(case["Q"], cuda), 100)
    assert e.value.code == la.ENOTSUP


@pytest.mark.parametrize("ctx", [3000, 40000])
def test_verify_round_head_dim_128(la, orc, synth, cuda, ctx):
    """A verify round at the reference geometry: the drafts' append (inside the attention kernel, in the last split
    of each kv head; at 40000 tokens that split also gives two tiles of attention to the others), the attention
    and the rollback; the cache bytes after the round are the oracle's, bit for bit."""
    m = 8
    case = synth.verify_case(74 + ctx % 7, ctx, m, q_heads=16, kv_heads=4, head_dim=128)
    cache = la.LayerCache(la.MODE_F16, 4, 128, ctx + 128, device=cuda)
    rope_np = la.rope_table(1e6, 0.5, 128, ctx + m + 1)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    out = cache.verify_round(dev(case["newK"], cuda), dev(case["newV"], cuda), dev(case["Q"], cuda), ctx,
                             rope=dev(rope_np.view(np.float16), cuda))
    la.sync()
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], ctx, rope=rope_np.view(np.float16))
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    assert rel_err(out.float().cpu().numpy(), orc.attention_f64(case["Q"], ctx, K, V, ctx + m)) < TOL
    logical = cache.logical(ctx + m)
    assert np.array_equal(logical["K"].view(np.uint16), K.view(np.uint16))
    assert np.array_equal(logical["V"].view(np.uint16), V.view(np.uint16))
    cache.truncate(ctx + 3)
    la.sync()
    v8, sc = orc.quantize_v8(V[:ctx + 3], ctx + 3)
    logical = cache.logical(ctx + 3)
    assert np.array_equal(logical["V8"], v8) and np.array_equal(logical["vscale"], sc)


def test_verify_round_c3_full_size(la, orc, synth, cuda):
    """Benchmark config 3 at full size through the round entry point: 131072 cached tokens (seed 2), 16 drafts
    appended with RoPE inside the attention kernel, verified causally. The output against exact fp64 and against
    the oracle's split-KV verify; the drafts' cache bytes (K, V, the int8 V of their block) bit-exact."""
    ctx, m = 131072, 16
    case = synth.verify_case(2, ctx, m)
    rope_np = la.rope_table(1e6, 1.0, 64, ctx + m + 1)
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx + m + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    out = cache.verify_round(dev(case["newK"], cuda), dev(case["newV"], cuda), dev(case["Q"], cuda), ctx,
                             rope=dev(rope_np.view(np.float16), cuda))
    la.sync()
    got = out.float().cpu().numpy()
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], ctx, rope=rope_np.view(np.float16))
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    assert rel_err(got, orc.attention_f64(case["Q"], ctx, K, V, ctx + m)) < TOL
    assert rel_err(got, orc.verify(case["Q"], K, V, ctx, splits=37)) < TOL_PAIR
    pool = cache.pool.cpu().numpy()
    table = cache.table.cpu().numpy()
    tail = la.decode_pool(pool, table, cache.layout, ctx + m)
    assert np.array_equal(tail["K"][ctx:], k_new.view(np.uint16))
    assert np.array_equal(tail["V"][ctx:], v_new.view(np.uint16))
    v8, sc = orc.quantize_v8(V, ctx + m)
    assert np.array_equal(tail["V8"][ctx:ctx + m], v8[ctx:ctx + m])
    assert np.array_equal(tail["vscale"][-1], sc[-1])


def test_refused_round_leaves_cache_unchanged(la, synth, cuda):
    """A verify round whose workspace is too small is refused (LFM3A_EWORKSPACE) before the drafts' append is
    launched: the cache bytes stay as they were."""
    import ctypes

    import torch

    ctx, m = 4000, 16
    case = synth.verify_case(71, ctx, m)
    cache = la.LayerCache(la.MODE_F16, 8, 64, ctx + m + 64, device=cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    la.sync()
    before = cache.pool.clone()
    splits = la.verify_splits(cache.layout, ctx, m)
    assert splits > 1
    small = torch.empty(256, dtype=torch.uint8, device=cuda)
    out = torch.zeros((m, 32, 64), dtype=torch.float16, device=cuda)
    nk, nv, q = dev(case["newK"], cuda), dev(case["newV"], cuda), dev(case["Q"], cuda)
    rc = la.lib().lfm3a_verify_round(ctypes.byref(cache.view), nk.data_ptr(), nv.data_ptr(), 0, None, None,
                                     q.data_ptr(), m, 32, ctx, 0, None, out.data_ptr(), small.data_ptr(), 256, splits,
                                     torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == la.EWORKSPACE
    la.sync()
    assert torch.equal(cache.pool, before)
    assert not out.any()
