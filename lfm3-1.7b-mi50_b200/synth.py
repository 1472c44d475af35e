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
