"""The prefix cache (host code in the library) against the reference's own tests and the CPU restatement.

- FNV-1a 64 of the restatement against the published FNV test vectors, then the library's salt and chain
  hashes against the restatement bit for bit.
- The reference's tests (internal/model/cache_test.go): chain hashes depend on salt and history; full
  blocks are evicted least recently used and never while pinned; a sliding block is reusable until the
  ring comes within the reuse margin; the conv ring never hands out slot 0.
- Random request streams (reuse, ensure, register with conv checkpoints, release, reset) through the
  library and the restatement side by side: every reuse result, block table and pool count agrees.
"""
import numpy as np
import pytest

from oracle import prefix as ref


def toks(seed: int) -> np.ndarray:
    return np.arange(seed, seed + 32, dtype=np.int32)


def test_fnv_published_vectors():
    assert ref.fnv1a64(b"") == 0xCBF29CE484222325
    assert ref.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert ref.fnv1a64(b"foobar") == 0x85944171F73967E8


def test_hashes_match_restatement(la):
    rng = np.random.default_rng(7)
    for salt in ("", "x", "user-42", "prefix"):
        assert la.prefix_salt(salt) == ref.salt_seed(salt)
    h = la.prefix_salt("s")
    for _ in range(50):
        block = rng.integers(-(2 ** 31), 2 ** 31, size=32, dtype=np.int64).astype(np.int32)
        want = ref.chain_hash(h, block)
        assert la.prefix_chain(h, block) == want
        h = want


def test_chain_hash_depends_on_history_and_salt(la):
    """cache_test.go:13-24."""
    a = la.prefix_chain(la.prefix_salt("x"), toks(1))
    assert a == la.prefix_chain(la.prefix_salt("x"), toks(1))
    assert a != la.prefix_chain(la.prefix_salt("y"), toks(1))
    assert la.prefix_chain(a, toks(2)) != la.prefix_chain(la.prefix_chain(la.prefix_salt("x"), toks(9)), toks(2))


def test_full_block_lru(la):
    """cache_test.go:26-54, through the sequence calls: a pool of two blocks, both cached by one request;
    while it pins them neither can be evicted; after it lets go, touching block 0 again makes block 1 the
    coldest, which the next allocation evicts and drops from the index."""
    pc = la.PrefixCache(2, 300, 4)
    prompt = np.concatenate([toks(1), toks(100), [7]]).astype(np.int32)
    s = pc.sequence("x")
    s.ensure(1)
    assert pc.free_blocks == 0
    for upto in (32, 64):   # a conv checkpoint at each block end, so either prefix is reusable
        _, ep = pc.alloc_conv()
        s.register(prompt, upto, ep)
    full, _ = s.blocks()
    other = pc.sequence("y")
    with pytest.raises(la.LFM3AError) as e:
        other.ensure(0)   # pinned blocks must not be evicted
    assert e.value.code == la.ENOSPACE
    other.close()
    s.close()   # releases both: block 0 then block 1 become evictable, block 0 the coldest
    warm = pc.sequence("x")
    assert warm.reuse(np.concatenate([toks(1), [5]]).astype(np.int32), window=32)[0] == 32
    warm.close()   # block 0 is now the most recently used
    fresh = pc.sequence("z")
    fresh.ensure(0)
    assert fresh.blocks()[0][0] == full[1]
    assert pc.cached_blocks == 1
    fresh.close()
    probe = pc.sequence("x")
    assert probe.reuse(prompt, window=32)[0] == 32   # block 0 stays cached, block 1 left the index
    probe.close()
    pc.close()


def test_lru_evicts_the_coldest(la):
    """cache_test.go:40-53: after touching block A, an allocation evicts B, and B leaves the index."""
    pc = la.PrefixCache(2, 300, 4)
    a_prompt = np.concatenate([toks(1), [0]]).astype(np.int32)
    b_prompt = np.concatenate([toks(50), [0]]).astype(np.int32)
    for prompt in (a_prompt, b_prompt):
        s = pc.sequence("x")
        s.ensure(0)
        _, ep = pc.alloc_conv()
        s.register(prompt, 32, ep)
        s.close()
    fa = pc.sequence("x")
    assert fa.reuse(a_prompt, window=32)[0] == 32   # A becomes the most recently used
    a_block = fa.blocks()[0][0]
    fa.close()
    s = pc.sequence("y")
    s.ensure(0)
    assert s.blocks()[0][0] != a_block   # B, the coldest, was evicted
    s.close()
    probe = pc.sequence("x")
    assert probe.reuse(b_prompt, window=32)[0] == 0
    probe.close()
    probe = pc.sequence("x")
    assert probe.reuse(a_prompt, window=32)[0] == 32
    probe.close()
    pc.close()


def test_slide_ring_validity(la):
    """cache_test.go:56-77."""
    pc = la.PrefixCache(1, 300, 4)
    b, ep = pc.alloc_slide()
    assert (b, ep) == (0, 0) and pc.slide_valid(ep)
    for _ in range(300 - ref.SLIDE_REUSE_MARGIN - 2):
        pc.alloc_slide()
    assert pc.slide_valid(ep)
    pc.alloc_slide()
    assert not pc.slide_valid(ep)
    assert not pc.slide_valid(-1)
    pc.close()


def test_conv_ring_skips_running_slot(la):
    """cache_test.go:79-102."""
    pc = la.PrefixCache(1, 300, 4)
    seen = set()
    for _ in range(9):
        s, ep = pc.alloc_conv()
        assert s != 0 and pc.conv_slot(ep) == s
        seen.add(s)
    assert len(seen) == 3
    _, first = pc.alloc_conv()
    for _ in range(3):
        pc.alloc_conv()
    assert not pc.conv_valid(first)
    pc.close()


@pytest.mark.parametrize("align", [1, 2])
@pytest.mark.parametrize("seed", range(8))
def test_random_streams_match_restatement(la, seed, align):
    """Requests sharing prefixes (few distinct prompts, random lengths), with conv checkpoints at chunk
    boundaries, random releases and an occasional reset, through both implementations."""
    rng = np.random.default_rng(seed)
    full_blocks, slide_blocks, conv_slots, window = 24, 160, 6, 64
    pc = la.PrefixCache(full_blocks, slide_blocks, conv_slots)
    oc = ref.Cache(full_blocks, slide_blocks, conv_slots)
    bases = [rng.integers(0, 50000, size=400).astype(np.int32) for _ in range(3)]
    live = []
    for _ in range(120):
        op = rng.random()
        if op < 0.55 or not live:
            base = bases[rng.integers(len(bases))]
            n = int(rng.integers(1, 300))
            prompt = base[:n].copy()
            if rng.random() < 0.3:
                prompt[rng.integers(n):] = rng.integers(0, 50000)   # diverge somewhere
            salt = "ab"[rng.integers(2)]
            s, o = pc.sequence(salt), ref.Seq(salt)
            got = s.reuse(prompt, window, align)
            want = ref.reuse(oc, o, list(prompt), window, align)
            assert got == want and got[0] % (32 * align) == 0
            ok = True
            try:
                s.ensure((n - 1) // 32)
            except la.LFM3AError as e:
                assert e.code == la.ENOSPACE
                ok = False
            assert ok == ref.ensure(oc, o, (n - 1) // 32)
            if ok:
                for upto in sorted({int(x) for x in rng.integers(0, n + 1, size=2)}):
                    slot, ep = pc.alloc_conv()
                    assert (slot, ep) == oc.alloc_conv()
                    s.register(prompt, upto, ep)
                    ref.register(oc, o, list(prompt), upto, ep)
            full, slide = s.blocks()
            assert list(full) == o.full and list(slide) == o.slide
            live.append((s, o))
        elif op < 0.95:
            s, o = live.pop(int(rng.integers(len(live))))
            s.release()
            ref.release(oc, o)
            s.close()
        else:
            pc.reset()
            oc.reset()
        assert pc.free_blocks == len(oc.free)
        assert pc.cached_blocks == len(oc.by_hash)
    for s, o in live:
        s.release()
        ref.release(oc, o)
        s.close()
    assert pc.free_blocks == len(oc.free)
    pc.close()
