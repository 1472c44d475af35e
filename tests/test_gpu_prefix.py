"""Prefix reuse on the device layout: two requests share pages of one layer pool through their own block
tables, as the reference's sequences share a per-layer pool (generate.go:222-295, engine.go:682-685).

Request A appends 150 tokens and hands its first four pages (128 tokens, two int8 V blocks) to the prefix
cache; request B starts with A's 128 tokens, reuses those pages (align 2: whole int8 V blocks) and appends
60 tokens of its own. Checked:
  - B's table points at A's four physical pages and its own pages are disjoint from them;
  - B's logical cache (K, V fp16, int8 V and scales) equals B computed alone, bit for bit;
  - A's four shared pages are unchanged by B's appends;
  - verify attention over B's table against the oracle (4e-3) and fp64 (2e-3), and the int8-PV prefill of
    B's own 60 tokens over the shared pages against the oracle (2e-2), all relative to the RMS.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


def test_shared_prefix_pages(la, orc, synth, cuda):
    rng = np.random.default_rng(11)
    pool_blocks = 24
    pc = la.PrefixCache(pool_blocks, 300, 4)
    base = la.LayerCache(la.MODE_F16, 8, 64, pool_blocks * 32, device=cuda, pool_blocks=pool_blocks)
    table_np = orc.rope_table(1e6, 1.0, 64, 512)
    rope = dev(table_np.view(np.float16), cuda)
    s = synth.Stream(11)

    def view(seq):
        full, _ = seq.blocks()
        table = np.zeros(pool_blocks, dtype=np.int32)
        table[:len(full)] = full
        return la.LayerCache(la.MODE_F16, 8, 64, pool_blocks * 32, device=cuda, block_table=dev(table, cuda),
                             pool=base)

    # Request A.
    toks_a = rng.integers(0, 50000, size=150).astype(np.int32)
    ka, va = s.normal_f16((150, 8, 64)), s.normal_f16((150, 8, 64))
    seq_a = pc.sequence("u")
    assert seq_a.reuse(toks_a, align=2) == (0, 0)
    seq_a.ensure((150 - 1) // 32)
    ca = view(seq_a)
    ca.append(dev(ka, cuda), dev(va, cuda), 0, rope=rope)
    _, ep = pc.alloc_conv()
    seq_a.register(toks_a, 128, ep)
    la.sync()
    a_shared = ca.logical(128)
    full_a = seq_a.blocks()[0]
    seq_a.release()

    # Request B: A's first 128 tokens, then 60 of its own.
    toks_b = np.concatenate([toks_a[:128], rng.integers(0, 50000, size=60).astype(np.int32)])
    kb, vb = s.normal_f16((60, 8, 64)), s.normal_f16((60, 8, 64))
    seq_b = pc.sequence("u")
    reused, _ = seq_b.reuse(toks_b, align=2)
    assert reused == 128
    seq_b.ensure((188 - 1) // 32)
    full_b = seq_b.blocks()[0]
    assert list(full_b[:4]) == list(full_a[:4])
    assert not set(full_b[4:].tolist()) & set(full_a[:4].tolist())
    cb = view(seq_b)
    cb.length = reused
    cb.append(dev(kb, cuda), dev(vb, cuda), reused, rope=rope)
    la.sync()

    K, V = orc.kv_append_f16(np.concatenate([ka[:128], kb]), np.concatenate([va[:128], vb]), 0, rope=table_np)
    v8, vs = orc.quantize_v8(V, 188)
    got = cb.logical(188)
    assert np.array_equal(got["K"].view(np.uint16), K.view(np.uint16))
    assert np.array_equal(got["V"].view(np.uint16), V.view(np.uint16))
    assert np.array_equal(got["V8"], v8)
    assert np.array_equal(got["vscale"].view(np.uint32), vs.view(np.uint32))
    after = ca.logical(128)
    for key in ("K", "V", "V8", "vscale"):
        assert np.array_equal(after[key], a_shared[key])

    # Attention over B's table.
    q = s.normal_f16((16, 32, 64))
    out = cb.verify(dev(q, cuda), 172)
    la.sync()
    o = out.float().cpu().numpy()
    assert rel_err(o, orc.verify(q, K, V, 172)) < 4e-3
    assert rel_err(o, orc.attention_f64(q, 172, K, V, 188)) < 2e-3
    qp = s.normal_f16((60, 32, 64))
    pf = cb.prefill(dev(qp, cuda), reused, exact=False)
    la.sync()
    assert rel_err(pf.float().cpu().numpy(), orc.prefill_i8pv(qp, reused, K, v8, vs)) < 2e-2
    seq_b.release()
    assert pc.free_blocks + pc.cached_blocks == pool_blocks
    pc.close()
