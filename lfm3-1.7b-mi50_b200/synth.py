"""Seeded synthetic inputs of the benchmark configurations.

Generator: splitmix64(seed) -> Box-Muller -> fp16 (round to nearest even). Output i of splitmix64 is
mix(seed + (i + 1) * 0x9E3779B97F4A7C15), so the stream vectorises; value pair j uses outputs 2j and
2j + 1: u1 = max(out >> 11, 1) * 2^-53, u2 = (out >> 11) * 2^-53, z = sqrt(-2 ln u1) (cos, sin)(2 pi u2).
Arrays are drawn row-major from one stream in the order K, V, new K, new V, Q.
"""
from __future__ import annotations

import os

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix(seed: int, first: int, count: int) -> np.ndarray:
    i = np.arange(first + 1, first + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + i * _GAMMA
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


class Stream:
    """A splitmix64 stream; normal_f16 draws consecutive values from it."""

    def __init__(self, seed: int):
        self.seed = seed
        self.pos = 0   # splitmix64 outputs consumed

    def normal(self, count: int, chunk: int = 1 << 22) -> np.ndarray:
        """count normal values (float64). Chunks are independent (the stream is indexed by position), so they
        are drawn on all host threads; the values do not depend on the chunking."""
        if count % 2:
            raise ValueError("draw an even number of values")
        out = np.empty(count, dtype=np.float64)
        base = self.pos
        self.pos += count

        def fill(done: int) -> None:
            n = min(chunk, count - done)
            raw = _splitmix(self.seed, base + done, n)
            u = (raw >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
            u1 = np.maximum(u[0::2], 2.0 ** -53)
            u2 = u[1::2]
            r = np.sqrt(-2.0 * np.log(u1))
            ang = 2.0 * np.pi * u2
            out[done:done + n:2] = r * np.cos(ang)
            out[done + 1:done + n:2] = r * np.sin(ang)

        starts = range(0, count, chunk)
        if count > chunk:
            from concurrent.futures import ThreadPoolExecutor

            with ThreadPoolExecutor(max_workers=min(len(starts), os.cpu_count() or 1)) as pool:
                list(pool.map(fill, starts))
        else:
            for done in starts:
                fill(done)
        return out

    def normal_f16(self, shape) -> np.ndarray:
        """fp16 values (as float16) of the requested shape."""
        n = int(np.prod(shape))
        return self.normal(n).astype(np.float32).astype(np.float16).reshape(shape)


def _normal_rows(seed: int, first: int, rows: int, row_stride: int, offset: int, width: int,
                 chunk_rows: int = 8192) -> np.ndarray:
    """Values first + r * row_stride + offset + [0, width) of a stream, r < rows, as float16 [rows][width]:
    the same numbers normal_f16 draws at those positions (offset, width and row_stride even), without the
    positions between them."""
    out = np.empty((rows, width), dtype=np.float16)

    def fill(r0: int) -> None:
        r1 = min(rows, r0 + chunk_rows)
        pos = (first + offset + np.arange(r0, r1, dtype=np.int64)[:, None] * row_stride +
               np.arange(0, width, 2, dtype=np.int64)[None, :]).reshape(-1)
        i = pos.astype(np.uint64) + np.uint64(1)   # output pos of the stream is mix(seed + (pos + 1) gamma)
        with np.errstate(over="ignore"):
            z = []
            for j in (i, i + np.uint64(1)):
                v = np.uint64(seed) + j * _GAMMA
                v = (v ^ (v >> np.uint64(30))) * _M1
                v = (v ^ (v >> np.uint64(27))) * _M2
                z.append(v ^ (v >> np.uint64(31)))
        u1 = np.maximum((z[0] >> np.uint64(11)).astype(np.float64) * (2.0 ** -53), 2.0 ** -53)
        u2 = (z[1] >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
        r = np.sqrt(-2.0 * np.log(u1))
        ang = 2.0 * np.pi * u2
        vals = np.empty((pos.size, 2), dtype=np.float64)
        vals[:, 0] = r * np.cos(ang)
        vals[:, 1] = r * np.sin(ang)
        out[r0:r1] = vals.reshape(r1 - r0, width).astype(np.float32).astype(np.float16)

    starts = range(0, rows, chunk_rows)
    if len(starts) > 1:
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(max_workers=min(len(starts), os.cpu_count() or 1)) as pool:
            list(pool.map(fill, starts))
    else:
        for r0 in starts:
            fill(r0)
    return out


def verify_case_heads(seed: int, ctx_len: int, m: int, h0: int, h1: int, q_heads: int = 32, kv_heads: int = 8,
                      head_dim: int = 64) -> dict:
    """kv heads [h0, h1) of verify_case(seed, ctx_len, m) (and their query heads), drawn without the others:
    a rank of the kv-head plan generates only its share. Bit-identical to slicing verify_case."""
    g = q_heads // kv_heads
    row = kv_heads * head_dim
    off, width = h0 * head_dim, (h1 - h0) * head_dim
    base = 0
    out = {}
    for name, rows in (("K", ctx_len), ("V", ctx_len), ("newK", m), ("newV", m)):
        out[name] = _normal_rows(seed, base, rows, row, off, width).reshape(rows, h1 - h0, head_dim)
        base += rows * row
    out["Q"] = _normal_rows(seed, base, m, q_heads * head_dim, g * off, g * width).reshape(m, g * (h1 - h0), head_dim)
    return out


def verify_case(seed: int, ctx_len: int, m: int, q_heads: int = 32, kv_heads: int = 8, head_dim: int = 64) -> dict:
    """Cache K, V [ctx_len][kv_heads][head_dim], drafts new K, new V [m][kv_heads][head_dim], Q [m][q_heads][head_dim]."""
    s = Stream(seed)
    return {
        "K": s.normal_f16((ctx_len, kv_heads, head_dim)),
        "V": s.normal_f16((ctx_len, kv_heads, head_dim)),
        "newK": s.normal_f16((m, kv_heads, head_dim)),
        "newV": s.normal_f16((m, kv_heads, head_dim)),
        "Q": s.normal_f16((m, q_heads, head_dim)),
    }


def prefill_case(seed: int, tokens: int, q_heads: int = 32, kv_heads: int = 8, head_dim: int = 64) -> dict:
    """Prompt K, V [tokens][kv_heads][head_dim] and Q [tokens][q_heads][head_dim] (config 4's draw order)."""
    s = Stream(seed)
    return {
        "K": s.normal_f16((tokens, kv_heads, head_dim)),
        "V": s.normal_f16((tokens, kv_heads, head_dim)),
        "Q": s.normal_f16((tokens, q_heads, head_dim)),
    }


def geometric_keep(seed: int, steps: int, p_stop: float = 0.3, cap: int = 16) -> np.ndarray:
    """Accepted lengths n = min(cap, X), P(X = k) = (1 - p_stop)^(k - 1) p_stop (config 5)."""
    s = Stream(seed ^ 0x5A5A5A5A)
    u = (_splitmix(s.seed, 0, steps) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    u = np.maximum(u, 2.0 ** -53)
    x = np.floor(np.log(u) / np.log(1.0 - p_stop)).astype(np.int64) + 1
    return np.minimum(x, cap)
