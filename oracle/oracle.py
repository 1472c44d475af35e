"""ctypes wrapper of the CPU restatement in oracle.cpp.

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it as
the checker. Parity status: unpinned against the reference itself (see oracle.h).
fp16 arrays travel as numpy float16 (bit-identical to the uint16 patterns the C side takes).
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_lib = None

_SIGS = {
    "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
    "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
    "orc_rope_table": (None, [ctypes.c_double, ctypes.c_double, _I, _I, _P]),
    "orc_kv_append_f16": (None, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "orc_kv_append_i8rec": (None, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "orc_quantize_v8": (None, [_P, _I, _I, _I, _P, _P]),
    "orc_quantize_p_u8": (None, [_P, _I, _I, _P, _P]),
    "orc_verify": (None, [_P, _I, _I, _I, _I, _P, _P, _I, _I, _P, _I, _P]),
    "orc_quantize_q": (None, [_P, ctypes.c_int64, _I, _I, _I, _P]),
    "orc_verify_i8rec": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _P, _I, _P]),
    "orc_prefill_i8rec": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _P]),
    "orc_prefill_i8rec_exact": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _P]),
    "orc_verify_partial": (None, [_P, _I, _I, _I, _I, _P, _P, _I, _I, _I, _I, _P]),
    "orc_combine": (None, [_P, _I, _I, _I, _P, _P]),
    "orc_attention_f64": (None, [_P, _I, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P]),
    "orc_prefill_i8pv": (None, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _I, _I, _P]),
    "orc_prefill_exact": (None, [_P, _I, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P]),
    "orc_q_norm_rope": (None, [_P, _I, _I, _I, ctypes.c_int64, _P, _P, _I, _P]),
    "orc_accept": (_I, [_P, _P, _I]),
    "orc_g128_exp": (ctypes.c_float, [ctypes.c_float]),
    "orc_g128_quantize": (None, [_P, ctypes.c_int64, _I, _I, _I, _P, _P]),
    "orc_g128_gemm": (None, [_P, _P, _P, _P, _I, _I, _I, _P, ctypes.c_int64, _P]),
    "orc_set_threads": (None, [_I]),
    "orc_get_threads": (_I, []),
}


def build() -> pathlib.Path:
    res = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + res.stdout + res.stderr)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def _c(a: np.ndarray | None, dtype=None):
    if a is None:
        return None, None
    a = np.ascontiguousarray(a, dtype=dtype) if dtype is not None else np.ascontiguousarray(a)
    return a, a.ctypes.data


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


def rope_table(theta: float, factor: float, head_dim: int, positions: int) -> np.ndarray:
    out = np.empty((positions, head_dim), dtype=np.float16)
    lib().orc_rope_table(theta, factor, head_dim, positions, out.ctypes.data)
    return out


def kv_append_f16(k, v, pos0: int, rope=None, knorm=None):
    n, h, d = k.shape
    k, kp = _c(k, np.float16)
    v, vp = _c(v, np.float16)
    rope, rp = _c(rope, np.float16)
    knorm, np_ = _c(knorm, np.float16)
    ko = np.empty_like(k)
    vo = np.empty_like(v)
    lib().orc_kv_append_f16(kp, vp, n, h, d, pos0, rp, np_, ko.ctypes.data, vo.ctypes.data)
    return ko, vo


def kv_append_i8rec(k, v, pos0: int, rope=None, knorm=None) -> np.ndarray:
    n, h, d = k.shape
    k, kp = _c(k, np.float16)
    v, vp = _c(v, np.float16)
    rope, rp = _c(rope, np.float16)
    knorm, np_ = _c(knorm, np.float16)
    rec = np.empty((n, h, 2 * d + 8), dtype=np.uint8)
    lib().orc_kv_append_i8rec(kp, vp, n, h, d, pos0, rp, np_, rec.ctypes.data)
    return rec


def quantize_v8(v, length: int | None = None):
    length = v.shape[0] if length is None else length
    _, h, d = v.shape
    v, vp = _c(v[:length], np.float16)
    nblk = (length + 63) // 64
    v8 = np.empty((nblk * 64, h, d), dtype=np.int8)
    sc = np.empty((nblk, h), dtype=np.float32)
    lib().orc_quantize_v8(vp, length, h, d, v8.ctypes.data, sc.ctypes.data)
    return v8, sc


def quantize_p_u8(p):
    p, pp = _c(p, np.float32)
    rows, cols = p.shape
    q = np.empty((rows, cols), dtype=np.uint8)
    sc = np.empty((rows,), dtype=np.float32)
    lib().orc_quantize_p_u8(pp, rows, cols, q.ctypes.data, sc.ctypes.data)
    return q, sc


def verify(q, K, V, ctx_len: int, window: int = 0, gate=None, splits: int = 1) -> np.ndarray:
    m, qh, d = q.shape
    kvh = K.shape[1]
    q, qp = _c(q, np.float16)
    K, kp = _c(K, np.float16)
    V, vp = _c(V, np.float16)
    gate, gp = _c(gate, np.float16)
    out = np.empty((m, qh, d), dtype=np.float32)
    lib().orc_verify(qp, m, qh, kvh, d, kp, vp, ctx_len, window, gp, splits, out.ctypes.data)
    return out


def quantize_q(q, q_heads: int | None = None, head_dim: int | None = None) -> np.ndarray:
    """prefill_attn.hip:120-135: q fp16 [T][q_heads][head_dim] (or [T][>= q_heads * head_dim] rows with
    q_heads, head_dim given) -> qbuf uint32 [T * q_heads][head_dim / 4 + head_dim / 32]."""
    q = np.ascontiguousarray(q, dtype=np.float16)
    t = q.shape[0]
    if q_heads is None:
        q_heads, head_dim = q.shape[1], q.shape[2]
    stride = int(np.prod(q.shape[1:]))
    out = np.empty((t * q_heads, head_dim // 4 + head_dim // 32), dtype=np.uint32)
    lib().orc_quantize_q(q.ctypes.data, stride, t, q_heads, head_dim, out.ctypes.data)
    return out


def dequantize_q(qbuf, head_dim: int) -> np.ndarray:
    """The float values a qbuf row stands for: int8 dims times their group scale, [rows][head_dim] float64."""
    qbuf = np.ascontiguousarray(qbuf, dtype=np.uint32)
    q8 = qbuf[:, :head_dim // 4].view(np.int8).reshape(qbuf.shape[0], head_dim).astype(np.float64)
    sc = qbuf[:, head_dim // 4:].view(np.float32).astype(np.float64)
    return q8 * np.repeat(sc, 32, axis=1)


def verify_i8rec(qbuf, m: int, q_heads: int, rec, ctx_len: int, window: int = 0, gate=None,
                 splits: int = 1) -> np.ndarray:
    """dspark.hip:1824-2185 over int8 records rec [ctx_len + m][kv_heads][2 * head_dim + 8] uint8 with the query
    rows qbuf (quantize_q of the m tokens) -> out [m][q_heads][head_dim] float32."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    kvh, rb = rec.shape[1], rec.shape[2]
    d = (rb - 8) // 2
    qbuf = np.ascontiguousarray(qbuf, dtype=np.uint32)
    gate, gp = _c(gate, np.float16)
    out = np.empty((m, q_heads, d), dtype=np.float32)
    lib().orc_verify_i8rec(qbuf.ctypes.data, m, q_heads, kvh, d, rec.ctypes.data, ctx_len, window, gp, splits,
                           out.ctypes.data)
    return out


def prefill_i8rec(qbuf, tokens: int, q_heads: int, rec, context: int, window: int = 0, splits: int = 1,
                  exact: bool = False) -> np.ndarray:
    """prefill_attn.hip:212-505 (exact: prefill_attn_exact.hip:173-344) over int8 records
    rec [context + tokens][kv_heads][2 * head_dim + 8] uint8 with the query rows qbuf (quantize_q of the tokens)
    -> out [tokens][q_heads][head_dim] float32."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    kvh, rb = rec.shape[1], rec.shape[2]
    d = (rb - 8) // 2
    qbuf = np.ascontiguousarray(qbuf, dtype=np.uint32)
    out = np.empty((tokens, q_heads, d), dtype=np.float32)
    fn = lib().orc_prefill_i8rec_exact if exact else lib().orc_prefill_i8rec
    fn(qbuf.ctypes.data, tokens, q_heads, kvh, d, rec.ctypes.data, context, window, splits, out.ctypes.data)
    return out


def dequantize_rec(rec) -> tuple[np.ndarray, np.ndarray]:
    """K and V float64 [tokens][kv_heads][head_dim] that int8 records stand for (int8 times its scale)."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    t, h, rb = rec.shape
    d = (rb - 8) // 2
    k8 = rec[..., :d].view(np.int8).astype(np.float64)
    ks = rec[..., d:d + 4].copy().view(np.float32).astype(np.float64)
    v8 = rec[..., d + 4:2 * d + 4].view(np.int8).astype(np.float64)
    vs = rec[..., 2 * d + 4:].copy().view(np.float32).astype(np.float64)
    return k8 * ks, v8 * vs


def verify_partial(q, K, V, kv_begin: int, kv_end: int, ctx_len: int, window: int = 0) -> np.ndarray:
    """Partial [m * q_heads][d + 2] (acc, max, sum) of the keys [kv_begin, kv_end); K/V by global position."""
    m, qh, d = q.shape
    kvh = K.shape[1]
    q, qp = _c(q, np.float16)
    K, kp = _c(K, np.float16)
    V, vp = _c(V, np.float16)
    part = np.empty((m * qh, d + 2), dtype=np.float32)
    lib().orc_verify_partial(qp, m, qh, kvh, d, kp, vp, kv_begin, kv_end, ctx_len, window, part.ctypes.data)
    return part


def combine(parts, head_dim: int, gate=None) -> np.ndarray:
    """Merge of partials [splits][rows][head_dim + 2] into [rows][head_dim] f32."""
    parts = np.ascontiguousarray(parts, dtype=np.float32)
    splits, rows = parts.shape[0], parts.shape[1]
    gate, gp = _c(gate, np.float16)
    out = np.empty((rows, head_dim), dtype=np.float32)
    lib().orc_combine(parts.ctypes.data, rows, splits, head_dim, gp, out.ctypes.data)
    return out


def attention_f64(q, qpos0: int, K, V, kv_len: int, window: int = 0, row_step: int = 1) -> np.ndarray:
    nq, qh, d = q.shape
    kvh = K.shape[1]
    q, qp = _c(q, np.float16)
    K, kp = _c(K, np.float16)
    V, vp = _c(V, np.float16)
    out = np.zeros((nq, qh, d), dtype=np.float32)
    lib().orc_attention_f64(qp, nq, qpos0, qh, kvh, d, kp, vp, kv_len, window, row_step, out.ctypes.data)
    return out


def prefill_i8pv(q, context: int, K, V8, vscale, window: int = 0, row_step: int = 1, splits: int = 1) -> np.ndarray:
    t, qh, d = q.shape
    kvh = K.shape[1]
    q, qp = _c(q, np.float16)
    K, kp = _c(K, np.float16)
    V8, v8p = _c(V8, np.int8)
    vscale, sp = _c(vscale, np.float32)
    out = np.zeros((t, qh, d), dtype=np.float32)
    lib().orc_prefill_i8pv(qp, t, context, qh, kvh, d, kp, v8p, sp, window, row_step, splits, out.ctypes.data)
    return out


def prefill_exact(q, context: int, K, V, window: int = 0, row_step: int = 1, splits: int = 1) -> np.ndarray:
    t, qh, d = q.shape
    kvh = K.shape[1]
    q, qp = _c(q, np.float16)
    K, kp = _c(K, np.float16)
    V, vp = _c(V, np.float16)
    out = np.zeros((t, qh, d), dtype=np.float32)
    lib().orc_prefill_exact(qp, t, context, qh, kvh, d, kp, vp, window, row_step, splits, out.ctypes.data)
    return out


def q_norm_rope(q, q_heads: int, head_dim: int, context: int, qnorm=None, rope=None) -> np.ndarray:
    """ops.hip:202-210. q: [T][>= q_heads * head_dim] fp16 rows; returns fp16 [T][q_heads][head_dim]."""
    q = np.ascontiguousarray(np.asarray(q, dtype=np.float16).reshape(q.shape[0], -1))
    t = q.shape[0]
    out = np.empty((t, q_heads, head_dim), dtype=np.float16)
    qn = None if qnorm is None else np.ascontiguousarray(np.asarray(qnorm).view(np.uint16))
    rp = None if rope is None else np.ascontiguousarray(np.asarray(rope).view(np.uint16))
    lib().orc_q_norm_rope(q.ctypes.data, t, q_heads, head_dim, q.shape[1], None if qn is None else qn.ctypes.data,
                          None if rp is None else rp.ctypes.data, context, out.ctypes.data)
    return out


def gate_mul(att, gate) -> np.ndarray:
    """ops.hip:254-264: the attention output rounded to fp16, times fp16(sigmoid(logit)) per (token, head),
    rounded to fp16 again (the product of two fp16 values is exact in fp32, so one rounding). att: fp32 or
    fp16 [T][QH][D]; gate: fp16 [T][>= QH]. sigmoid in fp32 with the host's expf."""
    g = np.asarray(gate, dtype=np.float16)[:, :att.shape[1]].astype(np.float32)
    s = (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32).astype(np.float16)
    return (np.asarray(att).astype(np.float16).astype(np.float32) * s.astype(np.float32)[..., None]).astype(np.float16)


def accept(best, tokens) -> int:
    best, bp = _c(best, np.int32)
    tokens, tp = _c(tokens, np.int32)
    return lib().orc_accept(bp, tp, tokens.shape[0])


# ------------------------------------------------------------------ W8A8 prefill GEMM (kernels/gemm.hip)
def g128_exp(x: float) -> float:
    return lib().orc_g128_exp(x)


def g128_quantize(x, k: int, gated: bool = False):
    """quantize_pack (gemm.hip:65-103). x: fp16 [rows][>= k] (>= 2k when gated). Returns q int8 [rows][k] and
    scales f32 [rows][k / 128], both row-major."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float16))
    rows = x.shape[0]
    q = np.empty((rows, k), dtype=np.int8)
    sc = np.empty((rows, k // 128), dtype=np.float32)
    lib().orc_g128_quantize(x.ctypes.data, x.shape[1], rows, k, int(gated), q.ctypes.data, sc.ctypes.data)
    return q, sc


def g128_gemm(qa, sa, qb, sb, residual=None) -> np.ndarray:
    """The W8A8 GEMM (gemm.hip:181-255) on row-major operands: qa [rows][k], sa [rows][k / 128], qb [outputs][k],
    sb [outputs][k / 128]; returns fp16 [rows][outputs]."""
    qa, ap = _c(qa, np.int8)
    qb, bp = _c(qb, np.int8)
    sa, sap = _c(sa, np.float32)
    sb, sbp = _c(sb, np.float32)
    rows, k = qa.shape
    outputs = qb.shape[0]
    res, rp = _c(residual, np.float16)
    out = np.empty((rows, outputs), dtype=np.float16)
    lib().orc_g128_gemm(ap, sap, bp, sbp, rows, outputs, k, rp, 0 if res is None else res.shape[1], out.ctypes.data)
    return out


def g128_pack(q, scales) -> tuple[np.ndarray, np.ndarray]:
    """Row-major int8 [rows][k] and f32 [rows][k / 128] into g128 tiles ([k/128][tiles][16384] bytes; row r, column c
    of a block at ((r/8)*8 + c/16)*128 + (r%8)*16 + c%16) and the scale layout [k/128][tiles * 128] (padding: 0, 1)."""
    q = np.asarray(q, dtype=np.int8)
    rows, k = q.shape
    tiles, groups = (rows + 127) // 128, k // 128
    qp = np.zeros((tiles * 128, k), dtype=np.int8)
    qp[:rows] = q
    # [tile][rg][r8][group][chunk][16] -> [group][tile][rg][chunk][r8][16]
    blk = qp.reshape(tiles, 16, 8, groups, 8, 16).transpose(3, 0, 1, 4, 2, 5)
    sp = np.ones((groups, tiles * 128), dtype=np.float32)
    sp[:, :rows] = np.asarray(scales, dtype=np.float32).T
    return np.ascontiguousarray(blk).reshape(-1).view(np.uint8), sp


def g128_unpack(packed, scales, rows: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of g128_pack: row-major int8 [rows][k] and f32 [rows][k / 128]."""
    tiles, groups = (rows + 127) // 128, k // 128
    blk = np.asarray(packed).view(np.int8).reshape(groups, tiles, 16, 8, 8, 16)
    q = blk.transpose(1, 2, 4, 0, 3, 5).reshape(tiles * 128, k)[:rows]
    sc = np.asarray(scales, dtype=np.float32).reshape(groups, tiles * 128)[:, :rows].T
    return np.ascontiguousarray(q), np.ascontiguousarray(sc)
