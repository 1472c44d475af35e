"""KV append / rollback / int8 V on the GPU against the oracle: bit-exact cache bytes and lengths."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def bits(a):
    return np.asarray(a).view(np.uint16)


def check_f16_cache(got, K, V, length, orc):
    assert np.array_equal(bits(got["K"][:length]), bits(K[:length]))
    assert np.array_equal(bits(got["V"][:length]), bits(V[:length]))
    v8, sc = orc.quantize_v8(V[:length], length)
    assert np.array_equal(got["V8"], v8)
    assert np.array_equal(got["vscale"].view(np.uint32), sc.view(np.uint32))


def test_append_then_rollback_c1(la, orc, synth, cuda):
    """Config 1: 1024 cached tokens, 8 drafts appended with RoPE theta 1e6 at 1024.., 3 rolled back."""
    import torch

    case = synth.verify_case(0, 1024, 8)
    cache = la.LayerCache(la.MODE_F16, 8, 64, 1024 + 64, device=cuda)
    rope = dev(la.rope_table(1e6, 1.0, 64, 1100).view(np.float16), cuda)
    cache.append(dev(case["K"], cuda), dev(case["V"], cuda), 0)
    cache.append(dev(case["newK"], cuda), dev(case["newV"], cuda), 1024, rope=rope)
    la.sync()
    table = orc.rope_table(1e6, 1.0, 64, 1100)
    k_new, v_new = orc.kv_append_f16(case["newK"], case["newV"], 1024, rope=table)
    K = np.concatenate([case["K"], k_new])
    V = np.concatenate([case["V"], v_new])
    check_f16_cache(cache.logical(1032), K, V, 1032, orc)
    cache.truncate(1029)
    la.sync()
    assert cache.length == 1029
    check_f16_cache(cache.logical(1029), K, V, 1029, orc)
    torch.cuda.synchronize()


def test_append_paged_norm_stride(la, orc, synth, cuda):
    """Permuted physical blocks, a k-norm, and K/V read out of a wider fused projection row."""
    import torch

    rng = np.random.default_rng(7)
    n_tok = 300
    s = synth.Stream(11)
    k = s.normal_f16((n_tok, 8, 64))
    v = s.normal_f16((n_tok, 8, 64))
    knorm = (1.0 + 0.25 * s.normal(64)).astype(np.float32).astype(np.float16)
    pages = (n_tok + 31) // 32
    perm = rng.permutation(40)[:pages].astype(np.int32)
    table = torch.from_numpy(perm).to(cuda)
    cache = la.LayerCache(la.MODE_F16, 8, 64, pages * 32, device=cuda, block_table=table, pool_blocks=40)
    stride = 3088
    f = np.zeros((n_tok, stride), dtype=np.float16)
    f[:, 2048:2048 + 512] = k.reshape(n_tok, 512)
    f[:, 2560:2560 + 512] = v.reshape(n_tok, 512)
    fd = dev(f, cuda)
    rope = dev(la.rope_table(1e6, 1.0, 64, 512).view(np.float16), cuda)
    # two appends that split a 64-token block: the second re-quantises the first's tail block
    cache.append(fd[:100, 2048:], fd[:100, 2560:], 0, rope=rope, k_norm=dev(knorm, cuda), token_stride=stride)
    cache.append(fd[100:, 2048:], fd[100:, 2560:], 100, rope=rope, k_norm=dev(knorm, cuda), token_stride=stride)
    la.sync()
    ko, vo = orc.kv_append_f16(k, v, 0, rope=orc.rope_table(1e6, 1.0, 64, 512), knorm=knorm)
    check_f16_cache(cache.logical(n_tok), ko, vo, n_tok, orc)


@pytest.mark.parametrize("new_len", [1, 63, 64, 65, 255])
def test_truncate_edges(la, orc, synth, cuda, new_len):
    s = synth.Stream(12)
    k = s.normal_f16((256, 8, 64))
    v = s.normal_f16((256, 8, 64))
    cache = la.LayerCache(la.MODE_F16, 8, 64, 256, device=cuda)
    cache.append(dev(k, cuda), dev(v, cuda), 0)
    cache.truncate(new_len)
    la.sync()
    check_f16_cache(cache.logical(new_len), k, v, new_len, orc)


def test_i8_records_reference_geometry(la, orc, synth, cuda):
    """The reference's own cache: 4 kv heads x 128 dims, 264-byte records, k-norm + RoPE (theta 1e6, factor 0.5)."""
    s = synth.Stream(13)
    n_tok = 77
    k = s.normal_f16((n_tok, 4, 128))
    v = s.normal_f16((n_tok, 4, 128))
    knorm = (1.0 + 0.25 * s.normal(128)).astype(np.float32).astype(np.float16)
    cache = la.LayerCache(la.MODE_I8REC, 4, 128, 96, device=cuda)
    rope_np = la.rope_table(1e6, 0.5, 128, 200)
    cache.append(dev(k, cuda), dev(v, cuda), 5, rope=dev(rope_np.view(np.float16), cuda), k_norm=dev(knorm, cuda))
    la.sync()
    got = cache.logical(5 + n_tok)["rec"][5:]
    want = orc.kv_append_i8rec(k, v, 5, rope=orc.rope_table(1e6, 0.5, 128, 200), knorm=knorm)
    assert got.shape == want.shape == (n_tok, 4, 264)
    assert np.array_equal(got, want)


def test_append_head_dim_128_norm_order(la, cuda):
    """The append's k-norm at head_dim 128 sums its squares in the reference's order (wave_sum, a pairwise tree over
    the 64 pairs d, d + 64): the golden rows, half of which round differently under a 32-lane butterfly, come out
    bit for bit."""
    import pathlib

    g = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "golden.npz")
    k = g["knorm_order_in"]
    cache = la.LayerCache(la.MODE_F16, 1, 128, k.shape[0] + 64, device=cuda)
    cache.append(dev(k, cuda), dev(k, cuda), 0, k_norm=dev(g["knorm128"], cuda))
    la.sync()
    got = cache.logical(k.shape[0])["K"]
    assert np.array_equal(got, g["knorm_order_out"].view(np.uint16))


def test_quantize_p_bitexact(la, orc, synth, cuda):
    s = synth.Stream(14)
    p = np.abs(s.normal(4096 * 64)).astype(np.float32).reshape(4096, 64)
    p *= np.float32(2.0) ** s.normal(4096).astype(np.float32).clip(-30, 10)[:, None].round()
    p[0] = 0
    p[1, :] = 0
    p[1, 9] = 3.0
    p[2] = np.arange(64, dtype=np.float32) / 2
    q, sc = la.quantize_p_u8(dev(p, cuda))
    la.sync()
    wq, wsc = orc.quantize_p_u8(p)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), wsc.view(np.uint32))


def test_accept_on_device(la, orc, cuda):
    import torch

    best = np.array([5, 6, 7, 9, 1, 2, 3, 4], dtype=np.int32)
    toks = np.array([4, 5, 6, 7, 8, 9, 9, 9], dtype=np.int32)
    state = torch.tensor([1024, 0, 0, 0], dtype=torch.int32, device=cuda)
    la.accept(dev(best, cuda), dev(toks, cuda), state)
    la.sync()
    commit = orc.accept(best, toks)
    assert state.cpu().tolist() == [1024 + commit, commit - 1, 8, commit]


@pytest.mark.parametrize("d", [64, 128])
def test_draft_rounds_append_rollback(la, orc, synth, cuda, d):
    """DSpark rounds on one cache: 5 drafts appended at the length, 2 kept (rollback of 3), repeated across
    64-token and page boundaries from an unaligned start; bytes and int8 V bit-exact after every round."""
    s = synth.Stream(14 + d)
    heads = 512 // d
    n0, rounds, drafts, keep = 61, 12, 5, 2
    total = n0 + rounds * keep + drafts
    k = s.normal_f16((total, heads, d))
    v = s.normal_f16((total, heads, d))
    kd = s.normal_f16((rounds, drafts, heads, d))
    vd = s.normal_f16((rounds, drafts, heads, d))
    table_np = orc.rope_table(1e6, 1.0, d, total + 8)
    rope = dev(table_np.view(np.float16), cuda)
    cache = la.LayerCache(la.MODE_F16, heads, d, total + 32, device=cuda)
    cache.append(dev(k[:n0], cuda), dev(v[:n0], cuda), 0, rope=rope)
    K, V = orc.kv_append_f16(k[:n0], v[:n0], 0, rope=table_np)
    length = n0
    for r in range(rounds):
        cache.append(dev(kd[r], cuda), dev(vd[r], cuda), length, rope=rope)
        kn, vn = orc.kv_append_f16(kd[r], vd[r], length, rope=table_np)
        K = np.concatenate([K[:length], kn])
        V = np.concatenate([V[:length], vn])
        la.sync()
        check_f16_cache(cache.logical(length + drafts), K, V, length + drafts, orc)
        length += keep
        cache.truncate(length)
        la.sync()
        check_f16_cache(cache.logical(length), K, V, length, orc)
