"""The C++ oracle against the golden vectors of tests/golden (an independent numpy restatement)."""
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "golden.npz"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def bits(a):
    return np.asarray(a).view(np.uint16)


def test_fp16_rounding(orc):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(size=20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
                        np.float32([0.0, -0.0, 65504.0, 65520.0, 1e-8, -6e-8, 2.0 ** -24, 3 * 2.0 ** -25, np.inf, -np.inf])])
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([orc.lib().orc_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(got, want)
    back = np.array([orc.lib().orc_f16_to_f32(int(b)) for b in want[:2000]], dtype=np.float32)
    assert np.array_equal(back, want[:2000].view(np.float16).astype(np.float32))


@pytest.mark.parametrize("name,theta,factor,d", [("rope_1e6_f1_d64", 1e6, 1.0, 64), ("rope_1e6_f05_d128", 1e6, 0.5, 128),
                                                 ("rope_1e4_f1_d128", 1e4, 1.0, 128)])
def test_rope_table(orc, g, name, theta, factor, d):
    pos = g["rope_1e6_f1_d64_pos"]
    table = orc.rope_table(theta, factor, d, int(pos.max()) + 1)
    assert np.array_equal(bits(table[pos]), bits(g[name]))


def test_append_f16_rope(orc, g):
    table = orc.rope_table(1e6, 1.0, 64, 1032)
    k, v = orc.kv_append_f16(g["c1_newK"], g["c1_newV"], 1024, rope=table)
    assert np.array_equal(bits(k), bits(g["c1_K_rope"]))
    assert np.array_equal(bits(v), bits(g["c1_newV"]))


def test_append_f16_norm_rope(orc, g):
    table = orc.rope_table(1e6, 1.0, 64, 1032)
    k, _ = orc.kv_append_f16(g["c1_newK"], g["c1_newV"], 1024, rope=table, knorm=g["knorm64"])
    assert np.array_equal(bits(k), bits(g["c1_K_norm_rope"]))


def test_append_i8_records(orc, g):
    table = orc.rope_table(1e6, 0.5, 128, 48)
    rec = orc.kv_append_i8rec(g["rec_k"], g["rec_v"], 40, rope=table, knorm=g["knorm128"])
    assert rec.shape[-1] == 264
    assert np.array_equal(rec, g["rec"])


def test_append_head_dim_128_norm_order(orc, g):
    """The k-norm's sum of squares at head_dim 128 follows the reference's wave_sum (a pairwise tree over its 64
    lanes, ops.hip:24-30,186-200): the fixture's first 16 rows round differently under a 32-lane butterfly."""
    k, _ = orc.kv_append_f16(g["knorm_order_in"], g["knorm_order_in"], 0, knorm=g["knorm128"])
    assert np.array_equal(bits(k), bits(g["knorm_order_out"]))


def test_v8_blocks(orc, g):
    v8, sc = orc.quantize_v8(g["v8_in"], 100)
    assert np.array_equal(v8, g["v8"])
    assert np.array_equal(sc.view(np.uint32), g["v8_scale"].view(np.uint32))
    assert np.all(sc[:, 3] == np.float32(1e-6))


def test_p_u8(orc, g):
    q, sc = orc.quantize_p_u8(g["p_in"])
    assert np.array_equal(q, g["p_q"])
    assert np.array_equal(sc.view(np.uint32), g["p_sc"].view(np.uint32))
    assert q[3].max() == 0 and q[4, 7] == 255


def test_accept(orc, g):
    best, toks = g["acc_best"], g["acc_tokens"]
    want = g["acc_commit"]
    assert orc.accept(best, toks) == want[0]
    assert orc.accept(best[:1], toks[:1]) == want[1]
    assert orc.accept(best, np.array([4, 0, 0, 0, 0, 0, 0, 0], dtype=np.int32)) == want[2]


def test_g128_exp(orc, g):
    got = np.array([orc.g128_exp(float(x)) for x in g["g128_exp_x"]], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), g["g128_exp_y"].view(np.uint32))
    # within 2 ulp of e^x over its finite range
    x = g["g128_exp_x"].astype(np.float64)
    live = (x >= -87) & (x < 88.5)
    rel = np.abs(got[live] / np.exp(x[live]) - 1.0)
    assert rel.max() < 2.5 * 2.0 ** -24


def test_g128_quantize(orc, g):
    q, sc = orc.g128_quantize(g["g128_x"], 384)
    assert np.array_equal(q, g["g128_qa"])
    assert np.array_equal(sc.view(np.uint32), g["g128_sa"].view(np.uint32))
    assert sc[3, 1] == 1.0 and not q[3, 128:256].any()


def test_g128_quantize_gated(orc, g):
    q, sc = orc.g128_quantize(g["g128_xg"], 256, gated=True)
    assert np.array_equal(q, g["g128_qg"])
    assert np.array_equal(sc.view(np.uint32), g["g128_sg"].view(np.uint32))


def test_g128_gemm(orc, g):
    out = orc.g128_gemm(g["g128_qa"], g["g128_sa"], g["g128_wq"], g["g128_ws"])
    assert np.array_equal(bits(out), bits(g["g128_out"]))
    out = orc.g128_gemm(g["g128_qa"], g["g128_sa"], g["g128_wq"], g["g128_ws"], residual=g["g128_resid"])
    assert np.array_equal(bits(out), bits(g["g128_out_resid"]))


def test_g128_tiles_round_trip(orc):
    rng = np.random.default_rng(5)
    q = rng.integers(-127, 128, size=(300, 384)).astype(np.int8)
    sc = rng.random((300, 3)).astype(np.float32)
    packed, sp = orc.g128_pack(q, sc)
    assert packed.size == 3 * 3 * 16384 and sp.shape == (3, 384)
    assert np.all(sp[:, 300:] == 1.0)
    q2, s2 = orc.g128_unpack(packed, sp, 300, 384)
    assert np.array_equal(q2, q) and np.array_equal(s2, sc)
    # row r, column c of group g, tile t sits at block (g, t), ((r/8)*8 + c/16)*128 + (r%8)*16 + c%16
    blk = packed.view(np.int8).reshape(3, 3, 16384)
    r, c = 133, 200
    assert blk[c // 128, r // 128, ((r % 128) // 8 * 8 + (c % 128) // 16) * 128 + (r % 8) * 16 + c % 16] == q[r, c]


def test_quantize_q(orc, g):
    """The oracle's query quantiser (prefill_attn.hip:120-135) against the golden rows: zero, tiny, large and tie
    values included."""
    q = g["q8_in"]
    got = orc.quantize_q(q.reshape(q.shape[0], 1, 128))
    assert np.array_equal(got, g["q8_out"])
