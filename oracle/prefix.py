"""CPU restatement of the reference's prefix cache, test infrastructure only: the checker for the library's
lfm3a_pcache_* / lfm3a_pseq_* / lfm3a_prefix_* entry points. Nothing in the product imports it.

Follows internal/model/cache.go (prefixCache, saltSeed, chainHash) and the sequence bookkeeping of
internal/model/generate.go:222-385 (reuse, ensureBlock, registerAt, release), line for line in behaviour,
in plain Python. FNV-1a 64 is the published algorithm (offset basis 0xcbf29ce484222325, prime 0x100000001b3),
the one Go's hash/fnv New64a implements; its published test vectors pin it (tests/test_prefix_cache.py).
"""
from __future__ import annotations

import struct

FNV_OFFSET = 0xCBF29CE484222325
FNV_PRIME = 0x100000001B3
MASK64 = (1 << 64) - 1
BLOCK_TOKENS = 32
SLIDE_REUSE_MARGIN = 128   # cache.go:12-16


def fnv1a64(data: bytes, h: int = FNV_OFFSET) -> int:
    for b in data:
        h = ((h ^ b) * FNV_PRIME) & MASK64
    return h


def salt_seed(salt: str) -> int:
    """cache.go:138-143: FNV-1a of "prefix-v1\\x00" then the salt."""
    return fnv1a64(salt.encode(), fnv1a64(b"prefix-v1\x00"))


def chain_hash(prev: int, tokens) -> int:
    """cache.go:145-154: FNV-1a of prev (u64 little endian) then each token (u32 little endian)."""
    toks = [int(t) & 0xFFFFFFFF for t in tokens]
    assert len(toks) == BLOCK_TOKENS
    return fnv1a64(struct.pack("<Q", prev) + struct.pack(f"<{BLOCK_TOKENS}I", *toks))


class Entry:
    __slots__ = ("hash", "full", "slide_epoch", "conv_epoch", "refs")

    def __init__(self, h, full, slide_epoch, conv_epoch=-1, refs=1):
        self.hash, self.full, self.slide_epoch, self.conv_epoch, self.refs = h, full, slide_epoch, conv_epoch, refs


class Cache:
    """cache.go:27-136. The LRU order is a Python list, least recently used first."""

    def __init__(self, full_blocks: int, slide_blocks: int, conv_slots: int):
        self.by_hash: dict[int, Entry] = {}
        self.free = list(range(full_blocks - 1, -1, -1))   # popped from the end: block 0 first
        self.lru: list[Entry] = []
        self.slide_blocks, self.slide_next = slide_blocks, 0
        self.conv_slots, self.conv_next = conv_slots - 1, 0

    def alloc_full(self):
        if self.free:
            return self.free.pop()
        if not self.lru:
            return None
        v = self.lru.pop(0)
        # cache.go:85 deletes v.hash unconditionally; after a reset a newer entry may hold that hash, so
        # both implementations here remove v only if the index still maps the hash to v.
        if self.by_hash.get(v.hash) is v:
            del self.by_hash[v.hash]
        return v.full

    def pin(self, e: Entry):
        if e.refs == 0:
            self.lru.remove(e)
        e.refs += 1

    def unpin(self, e: Entry):
        e.refs -= 1
        if e.refs == 0:
            self.lru.append(e)

    def alloc_slide(self):
        ep = self.slide_next
        self.slide_next += 1
        return ep % self.slide_blocks, ep

    def slide_valid(self, ep: int) -> bool:
        return ep >= 0 and self.slide_next - ep < self.slide_blocks - SLIDE_REUSE_MARGIN

    def alloc_conv(self):
        ep = self.conv_next
        self.conv_next += 1
        return ep % self.conv_slots + 1, ep

    def conv_valid(self, ep: int) -> bool:
        return ep >= 0 and self.conv_next - ep < self.conv_slots

    def conv_slot(self, ep: int) -> int:
        return ep % self.conv_slots + 1

    def reset(self):
        # cache.go:127-136 appends in Go map order (unspecified); both implementations here append the
        # freed blocks highest first, so the lowest is handed out first.
        self.free.extend(sorted((e.full for e in self.by_hash.values() if e.refs == 0), reverse=True))
        self.by_hash = {}
        self.lru = []


class Seq:
    """generate.go:50-61."""

    def __init__(self, salt: str = ""):
        self.hash = salt_seed(salt)
        self.registered = 0
        self.entries: list[Entry] = []
        self.private: list[int] = []
        self.full: list[int] = []
        self.slide: list[int] = []
        self.slide_epoch: list[int] = []
        self.released = False


def reuse(c: Cache, s: Seq, prompt, window: int, align: int = 1):
    """generate.go:222-279; returns (reused tokens, conv slot to restore or 0). align (not in the
    reference, whose per-token int8 records need none): the reused block count is a multiple of it."""
    limit = (len(prompt) - 1) // BLOCK_TOKENS if len(prompt) > 0 else 0
    chain = []
    h = s.hash
    for i in range(limit):
        h = chain_hash(h, prompt[i * BLOCK_TOKENS:(i + 1) * BLOCK_TOKENS])
        e = c.by_hash.get(h)
        if e is None:
            break
        chain.append(e)
    hit = 0
    for n in range(len(chain), 0, -1):
        if n % align != 0 or not c.conv_valid(chain[n - 1].conv_epoch):
            continue
        first = max(n * BLOCK_TOKENS - window + 1, 0)
        if all(c.slide_valid(chain[b].slide_epoch) for b in range(first // BLOCK_TOKENS, n)):
            hit = n
            break
    if hit == 0:
        return 0, 0
    for e in chain[:hit]:
        c.pin(e)
        s.entries.append(e)
        s.full.append(e.full)
        s.slide.append(e.slide_epoch % c.slide_blocks if e.slide_epoch >= 0 else 0)
        s.slide_epoch.append(e.slide_epoch)
        s.hash = e.hash
    s.registered = hit
    return hit * BLOCK_TOKENS, c.conv_slot(chain[hit - 1].conv_epoch)


def ensure(c: Cache, s: Seq, logical: int) -> bool:
    """generate.go:281-295."""
    while len(s.full) <= logical:
        f = c.alloc_full()
        if f is None:
            return False
        sl, ep = c.alloc_slide()
        s.full.append(f)
        s.slide.append(sl)
        s.slide_epoch.append(ep)
    return True


def register(c: Cache, s: Seq, tokens, upto: int, conv_epoch: int):
    """generate.go:346-373."""
    n = upto // BLOCK_TOKENS
    for i in range(s.registered, n):
        s.hash = chain_hash(s.hash, tokens[i * BLOCK_TOKENS:(i + 1) * BLOCK_TOKENS])
        e = c.by_hash.get(s.hash)
        if e is not None:
            c.pin(e)
            if e.full != s.full[i]:
                s.private.append(s.full[i])
            e.slide_epoch = s.slide_epoch[i]
        else:
            e = Entry(s.hash, s.full[i], s.slide_epoch[i])
            c.by_hash[s.hash] = e
        s.entries.append(e)
        if i == n - 1:
            e.conv_epoch = conv_epoch
    s.registered = max(s.registered, n)


def release(c: Cache, s: Seq):
    """generate.go:376-385."""
    if s.released:
        return
    for e in s.entries:
        c.unpin(e)
    c.free.extend(s.private)
    c.free.extend(s.full[s.registered:])
    s.released = True
