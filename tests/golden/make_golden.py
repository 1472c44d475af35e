"""Writes tests/golden/golden.npz: known-answer vectors for the bit-exact parts of the path, computed by
an independent numpy restatement of the reference lines (not by the C++ oracle they check).

The reference repository ships no golden vectors for these kernels, so these fixtures pin the oracle
to a second, separately written restatement of the same source lines:
  rope table       internal/model/engine.go:428-461 (buildRope)
  fp16 append      kernels/ops.hip:186-200 (norm_rotate), :236-251 (kv_write) into fp16 K/V
  int8 records     kernels/ops.hip:213-251 (quantize_pair, kv_write), 264-byte records at head_dim 128
  int8 V blocks    the same quantiser per (kv head, 64-token block)
  u8 P             kernels/prefill_attn.hip:305-331 (IEEE division in place of v_rcp_f32)
  int8 Q           kernels/prefill_attn.hip:120-135 (quantize_q: per 32-dim group, rint to nearest even)
  accept           kernels/dspark.hip:2851-2860
  W8A8 GEMM        kernels/gemm.hip:65-103 (quantize_pack, plain and gated) and :181-255 (gemm); every fp32
                   fma (the GEMM's group fold, the gate's exponential) emulated exactly with rationals
Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import math
import pathlib
from fractions import Fraction
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "lfm3-1.7b-mi50_b200"))
import synth  # noqa: E402  (the seeded generator of the benchmark inputs)

f32 = np.float32


def f16(x):
    return np.asarray(x, dtype=f32).astype(np.float16)


def rope_rows(theta, factor, d, positions):
    half, angles = d // 2, int(factor * d) // 2
    inv = np.zeros(half, dtype=f32)
    for i in range(angles):
        e = f32(2 * i) / f32(d)
        inv[i] = f32(1.0) / f32(math.pow(theta, float(e)))
    out = np.zeros((len(positions), d), dtype=np.float16)
    for r, p in enumerate(positions):
        t = f32(p)
        for i in range(half):
            f = float(f32(t * inv[i]))
            out[r, i] = np.float16(f32(math.cos(f)))
            out[r, half + i] = np.float16(f32(math.sin(f)))
    return out


def norm_rope(k, pos0, rope, knorm):
    """k: [n][h][d] float16 -> stored fp16; rope: full table [positions][d] or None; knorm [d] or None."""
    n, h, d = k.shape
    half, J = d // 2, d // 64
    x = k.astype(f32)
    a = np.stack([x[..., 32 * j:32 * j + 32] for j in range(J)], axis=-2)                 # [n][h][J][32]
    b = np.stack([x[..., half + 32 * j:half + 32 * j + 32] for j in range(J)], axis=-2)
    if knorm is not None:
        if d == 128:
            # ops.hip:186-200, 24-30: lane L of a 64-lane wave holds (L, L + 64); wave_sum adds the 64 lanes' a^2 + b^2
            # as a pairwise tree in natural order.
            v = x[..., :half] * x[..., :half] + x[..., half:] * x[..., half:]                 # [n][h][64]
            while v.shape[-1] > 1:
                v = v[..., 0::2] + v[..., 1::2]
            ss = v[..., 0]
        else:
            # head_dim 64 (no reference code): lane l of 32 holds (l, l + 32), butterfly o = 16 .. 1.
            lanes = a[..., 0, :] * a[..., 0, :] + b[..., 0, :] * b[..., 0, :]
            for o in (16, 8, 4, 2, 1):
                lanes = lanes + lanes[..., np.arange(32) ^ o]
            ss = lanes[..., 0]
        inv = f32(1.0) / np.sqrt(ss / f32(d) + f32(1e-5))
        w = knorm.astype(f32)
        wa = np.stack([w[32 * j:32 * j + 32] for j in range(J)])
        wb = np.stack([w[half + 32 * j:half + 32 * j + 32] for j in range(J)])
        a = f16((a * inv[..., None, None]) * wa).astype(f32)
        b = f16((b * inv[..., None, None]) * wb).astype(f32)
    if rope is not None:
        rows = rope[pos0:pos0 + n].astype(f32)                                             # [n][d]
        c = np.stack([rows[:, 32 * j:32 * j + 32] for j in range(J)], axis=-2)[:, None]    # [n][1][J][32]
        s = np.stack([rows[:, half + 32 * j:half + 32 * j + 32] for j in range(J)], axis=-2)[:, None]
        ra = f16(a * c - b * s).astype(f32)
        rb = f16(b * c + a * s).astype(f32)
        a, b = ra, rb
    out = np.zeros((n, h, d), dtype=np.float16)
    for j in range(J):
        out[..., 32 * j:32 * j + 32] = f16(a[..., j, :])
        out[..., half + 32 * j:half + 32 * j + 32] = f16(b[..., j, :])
    return out


def quant_half_away(x, inv):
    q = x.astype(f32) * inv
    q = np.where(q >= 0, q + f32(0.5), q - f32(0.5)).astype(f32)
    return np.trunc(np.clip(q, f32(-128), f32(127))).astype(np.int8)


def i8_records(kst, v):
    n, h, d = kst.shape
    rec = np.zeros((n, h, 2 * d + 8), dtype=np.uint8)
    for part, src in enumerate((kst.astype(f32), v.astype(f32))):
        amax = np.abs(src).max(axis=-1)
        scale = np.maximum(amax / f32(127), f32(1e-6)).astype(f32)
        inv = (f32(1) / scale).astype(f32)
        q = quant_half_away(src, inv[..., None])
        off = part * (d + 4)
        rec[..., off:off + d] = q.view(np.uint8)
        rec[..., off + d:off + d + 4] = scale[..., None].view(np.uint8).reshape(n, h, 4)
    return rec


def v8_blocks(v, length):
    _, h, d = v.shape
    nblk = (length + 63) // 64
    v8 = np.zeros((nblk * 64, h, d), dtype=np.int8)
    sc = np.zeros((nblk, h), dtype=f32)
    for b in range(nblk):
        t0, t1 = 64 * b, min(length, 64 * b + 64)
        blk = v[t0:t1].astype(f32)
        amax = np.abs(blk).max(axis=(0, 2))
        scale = np.maximum(amax / f32(127), f32(1e-6)).astype(f32)
        inv = (f32(1) / scale).astype(f32)
        sc[b] = scale
        v8[t0:t1] = quant_half_away(blk, inv[None, :, None])
    return v8, sc


def p_u8(p):
    pm = p.max(axis=1).astype(f32)
    inv = (f32(255) / np.maximum(pm, f32(1e-30))).astype(f32)
    x = (p * inv[:, None]).astype(f32)
    q = np.clip(np.rint(x), 0, 255).astype(np.uint8)
    return q, (pm * f32(1.0 / 255.0)).astype(f32)


def quantize_q(q):
    """q: [rows][d] float16 -> dwords [rows][d/4 + d/32]: the int8 dims packed in byte order, then the scales."""
    rows, d = q.shape
    x = q.astype(f32).reshape(rows, d // 32, 32)
    amax = np.abs(x).max(axis=2)
    scale = np.maximum(amax / f32(127.0), f32(1e-20)).astype(f32)
    inv = (f32(1.0) / scale).astype(f32)
    qi = np.rint((x * inv[:, :, None]).astype(f32)).astype(np.int64).reshape(rows, d)
    by = (qi & 0xFF).astype(np.uint8)
    out = np.zeros((rows, d // 4 + d // 32), dtype=np.uint32)
    out[:, :d // 4] = by.view(np.uint32).reshape(rows, d // 4)
    out[:, d // 4:] = scale.view(np.uint32)
    return out


def accept(best, tokens):
    acc = 0
    for t in range(len(tokens) - 1):
        if best[t] != tokens[t + 1]:
            break
        acc += 1
    return acc + 1


def fma32(a, b, c):
    """fmaf on float32 values: the exact a * b + c rounded once to float32 (ties to even)."""
    return round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def g128_exp_one(x):
    """e^x with the gated quantiser's steps: Cody-Waite reduction and degree-7 Taylor Horner, as fused
    multiply-adds (fma32), 2^n as two power-of-two factors."""
    x = f32(x)
    if np.isnan(x):
        return x
    if not x < f32(88.5):
        return f32(np.inf)
    if x < f32(-87.0):
        return f32(0.0)
    n = f32(np.rint(f32(x * f32(1.44269502))))
    r = fma32(-n, f32(1.42860677e-6), fma32(-n, f32(0.693145751953125), x))
    p = f32(1.98412701e-4)
    for c in (1.38888892e-3, 8.33333377e-3, 4.16666679e-2, 1.66666672e-1, 0.5, 1.0, 1.0):
        p = fma32(r, p, f32(c))
    ni = int(n)
    n1 = int(ni / 2)
    n2 = ni - n1
    f1 = np.array([(n1 + 127) << 23], dtype=np.uint32).view(f32)[0]
    f2 = np.array([(n2 + 127) << 23], dtype=np.uint32).view(f32)[0]
    return f32(f32(p * f1) * f2)


def g128_exp(x):
    x = np.asarray(x, dtype=f32)
    return np.array([g128_exp_one(v) for v in x.reshape(-1)], dtype=f32).reshape(x.shape)


def g128_quantize(x, k, gated):
    x = np.asarray(x, dtype=np.float16).astype(f32)
    v = x[:, :k]
    if gated:
        v = (v / (f32(1.0) + g128_exp(-v))) * x[:, k:2 * k]
    rows, groups = v.shape[0], k // 128
    vg = v.reshape(rows, groups, 128)
    m = np.abs(vg).max(axis=2)
    scale = np.where(m > 0, m / f32(127.0), f32(1.0)).astype(f32)
    inv = (f32(1.0) / scale).astype(f32)
    q = np.rint(np.clip(vg * inv[:, :, None], f32(-127.0), f32(127.0))).astype(np.int8)
    return q.reshape(rows, k), scale


def round_f32(fr):
    """Fraction -> the nearest float32, ties to even (normal range)."""
    if fr == 0:
        return f32(0.0)
    sign, a = (-1 if fr < 0 else 1), abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length() - 24
    while a / Fraction(2) ** e >= 2 ** 24:
        e += 1
    while a / Fraction(2) ** e < 2 ** 23:
        e -= 1
    q = round(a / Fraction(2) ** e)          # round() of a Fraction: half to even
    return f32(sign * q * 2.0 ** e)


def g128_gemm(qa, sa, qb, sb, residual):
    rows, k = qa.shape
    outputs, groups = qb.shape[0], k // 128
    s = np.einsum("mgi,ngi->mng", qa.reshape(rows, groups, 128).astype(np.int64),
                  qb.reshape(outputs, groups, 128).astype(np.int64))
    out = np.empty((rows, outputs), dtype=np.float16)
    for m in range(rows):
        for n in range(outputs):
            acc = f32(0.0)
            for gi in range(groups):
                t = f32(f32(s[m, n, gi]) * sb[n, gi])
                acc = round_f32(Fraction(float(t)) * Fraction(float(sa[m, gi])) + Fraction(float(acc)))
            if residual is not None:
                acc = f32(acc + f32(residual[m, n]))
            out[m, n] = np.float16(acc)
    return out


def main():
    g = {}
    # RoPE tables: the benchmark's (theta 1e6, all 32 pairs, D 64) and the reference model's two.
    pos = np.array([0, 1, 2, 31, 1023, 1024, 1031, 32767, 32783, 131071, 131087])
    g["rope_1e6_f1_d64_pos"] = pos
    g["rope_1e6_f1_d64"] = rope_rows(1e6, 1.0, 64, pos)
    g["rope_1e6_f05_d128"] = rope_rows(1e6, 0.5, 128, pos)
    g["rope_1e4_f1_d128"] = rope_rows(1e4, 1.0, 128, pos)

    # fp16 append, config 1 (seed 0): 8 drafts at positions 1024.. with RoPE theta 1e6.
    case = synth.verify_case(0, 1024, 8)
    table = rope_rows(1e6, 1.0, 64, np.arange(1032))
    g["c1_newK"], g["c1_newV"] = case["newK"], case["newV"]
    g["c1_K_rope"] = norm_rope(case["newK"], 1024, table, None)
    # Same drafts with a k-norm weight vector.
    s = synth.Stream(100)
    knorm64 = f16(1.0 + 0.25 * s.normal(64))
    g["knorm64"] = knorm64
    g["c1_K_norm_rope"] = norm_rope(case["newK"], 1024, table, knorm64)

    # Reference-geometry int8 records: 16/4/128, theta 1e6 factor 0.5, 5 tokens at position 40.
    s = synth.Stream(101)
    k128 = s.normal_f16((5, 4, 128))
    v128 = s.normal_f16((5, 4, 128))
    knorm128 = f16(1.0 + 0.25 * s.normal(128))
    table128 = rope_rows(1e6, 0.5, 128, np.arange(48))
    g["rec_k"], g["rec_v"], g["knorm128"] = k128, v128, knorm128
    g["rec"] = i8_records(norm_rope(k128, 40, table128, knorm128), v128)

    # The k-norm's sum of squares at head_dim 128 in the reference's order (a pairwise tree over its 64 lanes): rows
    # picked so that 16 of them round to other fp16 outputs under the butterfly order of a 32-lane warp (lane l
    # holding dims l, l + 32, l + 64, l + 96, o = 16 .. 1), and 16 that do not.
    s = synth.Stream(104)
    cand = s.normal_f16((16384, 1, 128))
    want = norm_rope(cand, 0, None, knorm128)
    x = cand[:, 0].astype(f32)
    lanes = (x[:, 0:32] * x[:, 0:32] + x[:, 64:96] * x[:, 64:96]) + (x[:, 32:64] * x[:, 32:64] + x[:, 96:] * x[:, 96:])
    for o in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, np.arange(32) ^ o]
    inv = f32(1.0) / np.sqrt(lanes[:, 0] / f32(128) + f32(1e-5))
    other = f16((x * inv[:, None]) * knorm128.astype(f32))
    differs = np.any(other != want[:, 0], axis=1)
    assert differs.sum() >= 16
    pick = np.concatenate([np.nonzero(differs)[0][:16], np.nonzero(~differs)[0][:16]])
    g["knorm_order_in"] = cand[pick]
    g["knorm_order_out"] = want[pick]

    # int8 V per 64-token block: 100 tokens (one full block, one partial), a zero head to hit the floor.
    s = synth.Stream(102)
    vq = s.normal_f16((100, 8, 64))
    vq[:, 3, :] = 0
    g["v8_in"] = vq
    g["v8"], g["v8_scale"] = v8_blocks(vq, 100)

    # u8 P rows: random, exact ties at .5 after scaling, an all-zero row, a single spike.
    s = synth.Stream(103)
    p = np.abs(s.normal(16 * 64)).astype(f32).reshape(16, 64)
    p[3] = 0
    p[4] = 0
    p[4, 7] = 1.0
    p[5] = np.arange(64, dtype=f32) / f32(2.0)       # pm = 31.5, inv = 255/31.5
    p[6] = f32(2.0) ** -40 * (np.arange(64, dtype=f32) + 1)
    g["p_in"] = p
    g["p_q"], g["p_sc"] = p_u8(p)

    # int8 Q rows (reference geometry, head_dim 128): random, an all-zero row, tiny values, a large value,
    # and values that land on .5 after scaling (ties to even).
    s = synth.Stream(105)
    q8 = s.normal_f16((12, 128))
    q8[1] = 0
    q8[2] = (q8[2].astype(f32) * f32(3e-5)).astype(np.float16)
    q8[3, 5] = np.float16(60000.0)
    q8[4, :32] = np.float16(0.5)
    q8[4, 0] = np.float16(127.0)
    q8[4, 1] = np.float16(2.5)
    g["q8_in"] = q8
    g["q8_out"] = quantize_q(q8)

    # accept
    best = np.array([5, 6, 7, 9, 1, 2, 3, 4], dtype=np.int32)
    toks = np.array([4, 5, 6, 7, 8, 9, 9, 9], dtype=np.int32)
    g["acc_best"], g["acc_tokens"] = best, toks
    g["acc_commit"] = np.array([accept(best, toks), accept(best[:1], toks[:1]), accept(best, np.array([4, 0, 0, 0, 0, 0, 0, 0]))])

    # W8A8 GEMM: 40 activation rows (ragged against the 128-row tile) x 384 inputs (3 groups) against 72
    # weight rows, with an all-zero group (scale 1), an exact .5 tie, and a residual; gated activations with
    # gate values past both clamps of the exponential.
    s = synth.Stream(104)
    x = s.normal_f16((40, 384))
    x[3, 128:256] = 0
    x[5, :128] = np.float16(0.25)
    x[5, 0] = np.float16(127.0 * 0.25 * 2 / 3)      # a value that lands near a .5 after scaling
    wq = np.clip(np.rint(s.normal(72 * 384) * 40.0), -127, 127).astype(np.int8).reshape(72, 384)
    ws = f16(np.abs(s.normal(72 * 3)) * 0.01 + 1e-3).astype(f32).reshape(72, 3)
    resid = s.normal_f16((40, 72))
    qa, sa = g128_quantize(x, 384, False)
    g["g128_x"], g["g128_qa"], g["g128_sa"] = x, qa, sa
    g["g128_wq"], g["g128_ws"], g["g128_resid"] = wq, ws, resid
    g["g128_out"] = g128_gemm(qa, sa, wq, ws, None)
    g["g128_out_resid"] = g128_gemm(qa, sa, wq, ws, resid)
    xg = s.normal_f16((24, 512))
    xg[0, :256] = np.float16(-100.0)
    xg[1, :256] = np.float16(95.0)
    xg[2, :256] = (np.arange(256) - 128).astype(np.float16)
    g["g128_xg"] = xg
    g["g128_qg"], g["g128_sg"] = g128_quantize(xg, 256, True)
    ex = np.concatenate([np.linspace(-90, 90, 721, dtype=f32), f32([-87.0, -86.99, 88.49, 88.5, 0.0, -0.0])])
    g["g128_exp_x"], g["g128_exp_y"] = ex, g128_exp(ex)

    np.savez_compressed(HERE / "golden.npz", **g)
    print("wrote", HERE / "golden.npz", sum(v.nbytes for v in g.values()), "bytes raw")


if __name__ == "__main__":
    main()
