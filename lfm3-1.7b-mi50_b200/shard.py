"""Sharding of one layer's KV cache over the GPUs of one node (one process per GPU).

Two plans, both with no collective inside the attention itself:

heads  Rank r owns kv heads [r * KVH / N, (r + 1) * KVH / N) of the whole sequence and their 4x query heads.
       Append, verify and prefill stay local; the per-rank outputs [m][QH / N][D] are all-gathered and laid
       side by side (query head qh lives on rank qh // (QH / N)).
seq    Rank r owns a contiguous run of 64-token blocks of the sequence (whole int8 V quantisation blocks, so
       no block's int8 copy spans two ranks); the last rank also holds the tail and the drafts. Each rank
       computes the log-sum-exp partial (acc, max, sum) of its keys (lfm3a_verify_partial); the partials
       [N][rows][D + 2] are all-gathered and merged (lfm3a_combine).

The reference engine runs one GPU; this split is the B200 build's own (the partial and merge arithmetic are
the reference's split-KV partials and combine_phase, dspark.hip:2100-2120, 2134-2185).
"""
from __future__ import annotations

RUN_TOKENS = 64   # granularity of the seq plan: the int8 V block (two 32-token pages)


def head_range(world: int, rank: int, kv_heads: int) -> tuple[int, int]:
    """kv heads [h0, h1) of this rank under the heads plan."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} kv heads do not split over {world} ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def query_head_range(world: int, rank: int, kv_heads: int, q_heads: int) -> tuple[int, int]:
    """Query heads [qh0, qh1) that read this rank's kv heads (grouped-query attention)."""
    h0, h1 = head_range(world, rank, kv_heads)
    group = q_heads // kv_heads
    return h0 * group, h1 * group


def seq_range(world: int, rank: int, ctx_len: int, m: int) -> tuple[int, int]:
    """Token range [kv_begin, kv_end) of this rank under the seq plan: equal runs of whole 64-token blocks of
    the ctx_len cached tokens, the last rank also holding the m drafts (positions ctx_len .. ctx_len + m - 1).
    A rank may hold no blocks when the context is short; its range is then empty (kv_begin == kv_end)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    if ctx_len < 0 or m < 0:
        raise ValueError("negative length")
    blocks = (ctx_len + RUN_TOKENS - 1) // RUN_TOKENS
    b0 = blocks * rank // world
    b1 = blocks * (rank + 1) // world
    begin = min(b0 * RUN_TOKENS, ctx_len)
    end = min(b1 * RUN_TOKENS, ctx_len)
    if rank == world - 1:
        end = ctx_len + m
    return begin, end


def assemble_heads(parts):
    """[N][m][QH / N][D] per-rank outputs (heads plan) -> [m][QH][D]."""
    import numpy as np

    if hasattr(parts, "permute"):   # torch tensor
        n, m, qh, d = parts.shape
        return parts.permute(1, 0, 2, 3).reshape(m, n * qh, d)
    parts = np.asarray(parts)
    n, m, qh, d = parts.shape
    return parts.transpose(1, 0, 2, 3).reshape(m, n * qh, d)
