"""The C-ABI library on CPU: it loads, exports every symbol include/lfm3attn.h declares, and its host-side
logic (layouts, RoPE table, argument checks) behaves. No kernel runs here."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "lfm3attn.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lfm3a_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported(la):
    names = declared_functions()
    assert len(names) >= 15
    handle = ctypes.CDLL(str(la.LIB_PATH))
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, missing
    assert set(names) <= set(la.SIGNATURES), set(names) - set(la.SIGNATURES)


def test_version_and_strings(la):
    assert la.lib().lfm3a_version() == 1
    assert la.lib().lfm3a_strerror(-1) == b"invalid argument"
    assert la.lib().lfm3a_strerror(-7).startswith(b"a kernel gave up")


@pytest.mark.parametrize("mode,h,d,head,block", [(0, 8, 64, 10368, 82944), (0, 4, 128, 20608, 82432),
                                                 (1, 4, 128, 264, 33792), (1, 8, 64, 136, 34816)])
def test_layouts(la, mode, h, d, head, block):
    lay = la.layout(mode, h, d)
    assert (lay.head_bytes, lay.block_bytes) == (head, block)
    assert lay.head_bytes % 128 == 0 or mode == 1


def test_layout_rejects(la):
    with pytest.raises(la.LFM3AError) as e:
        la.layout(0, 8, 96)
    assert e.value.code == la.ENOTSUP
    with pytest.raises(la.LFM3AError):
        la.layout(0, 8, 64, block_tokens=16)
    with pytest.raises(la.LFM3AError):
        la.layout(7, 8, 64)


@pytest.mark.parametrize("theta,factor,d", [(1e6, 1.0, 64), (1e6, 0.5, 128), (1e4, 1.0, 128)])
def test_rope_table_matches_oracle(la, orc, theta, factor, d):
    n = 4096
    got = la.rope_table(theta, factor, d, n)
    want = orc.rope_table(theta, factor, d, n).view(np.uint16)
    assert np.array_equal(got, want)


def test_argument_checks_without_device(la):
    lib = la.lib()
    view = la.KvView(None, None, 0, la.layout(0, 8, 64))
    assert lib.lfm3a_kv_append(ctypes.byref(view), None, None, 0, 0, 1, None, None, None) == la.EINVAL
    good = la.KvView(64, 64, 10, la.layout(0, 8, 64))
    bad_geom = la.KvView(64, 64, 10, la.layout(0, 4, 128))
    # head_dim 128 is served for up to 16 verified tokens (verify_m64_kernel<128>); more is refused on the host
    assert lib.lfm3a_verify_attention(ctypes.byref(bad_geom), 64, 17, 16, 100, 0, None, 64, None, 0, 1, None) == la.ENOTSUP
    assert lib.lfm3a_verify_attention(ctypes.byref(good), 64, 16, 16, 100, 0, None, 64, None, 0, 1, None) == la.ENOTSUP
    assert lib.lfm3a_verify_attention(ctypes.byref(good), 64, 40, 32, 100, 0, None, 64, None, 0, 1, None) == la.EINVAL
    assert lib.lfm3a_verify_attention(ctypes.byref(good), 64, 16, 32, 1000, 0, None, 64, None, 0, 4, None) == la.EINVAL
    assert lib.lfm3a_verify_attention(ctypes.byref(good), 64, 16, 32, 1000, 0, None, 64, 64, 16, 4, None) == la.EWORKSPACE
    assert lib.lfm3a_verify_partial(ctypes.byref(good), 64, 16, 32, 500, 400, 1000, 0, 64, None, 0, 1, None) == la.EINVAL
    assert lib.lfm3a_combine(None, 4, 2, 64, 0, 0, None, 64, None) == la.EINVAL
    assert lib.lfm3a_kv_truncate(ctypes.byref(good), -1, None) == la.EINVAL
    assert b"negative" in lib.lfm3a_last_error()
    # the host-buffer round checks its buffers before any copy: no host input, a misaligned device staging buffer
    assert lib.lfm3a_verify_round_host(ctypes.byref(good), None, 64, None, None, 16, 32, 100, 0, None, 64, 64, None,
                                       0, 1, None, 0) == la.EINVAL
    assert lib.lfm3a_verify_round_host(ctypes.byref(good), 64, 72, None, None, 16, 32, 100, 0, None, 64, 64, None,
                                       0, 1, None, 0) == la.EINVAL
    assert b"aligned" in lib.lfm3a_last_error()
    lay = la.layout(0, 8, 64)
    view_bad_stride = la.KvView(64, 64, 10, la.KvLayout(0, 8, 64, 32, 10000, 80000))
    assert lib.lfm3a_kv_truncate(ctypes.byref(view_bad_stride), 5, None) == la.EINVAL
    assert lay.head_bytes == 10368


def test_split_choice(la):
    lay = la.layout(0, 8, 64)
    assert la.verify_splits(lay, 32768, 16, 0, 148) == 37
    assert la.verify_splits(lay, 131072, 16, 0, 148) == 37
    # one kv head (a GPU's share on eight): 296 splits would stream 443 keys each, 148 stream 886
    one = la.layout(0, 1, 64)
    assert la.verify_splits(one, 131072, 16, 0, 148) == 148
    assert la.verify_splits(la.layout(0, 2, 64), 131072, 16, 0, 148) == 148
    assert la.verify_splits(la.layout(0, 4, 64), 131072, 16, 0, 148) == 74
    assert la.verify_splits(lay, 8192, 16, 0, 148) == 32   # mid contexts keep two per SM
    assert la.verify_splits(lay, 100, 8, 0, 148) == 1
    assert la.verify_splits(lay, 20, 8, 0, 148) == 1
    assert la.verify_splits(lay, 1024, 8, 0, 148) == 4     # 128-key tiles for m <= 16
    assert la.verify_splits(lay, 1024, 32, 0, 148) == 8    # 64-key tiles above
    ws = la.lib().lfm3a_verify_workspace_bytes(16, 32, 64, 37)
    assert ws == 16 * 32 * 37 * 66 * 4


def test_synth_generator_is_deterministic(synth):
    a = synth.Stream(3).normal_f16((1000,))
    s = synth.Stream(3)
    b = np.concatenate([s.normal_f16((400,)), s.normal_f16((600,))])
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    z = synth.Stream(0).normal(200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    keep = synth.geometric_keep(4, 256)
    assert keep.min() >= 1 and keep.max() <= 16 and 2.5 < keep.mean() < 4.0


def test_prefill_split_choice(la):
    """Chunks that fill one wave of two CTAs per SM run unsplit; short chunks over long contexts split into
    the count with the least modelled time (whole waves, 2 tiles of fixed cost per CTA), each split with at
    least 8 key tiles of the shortest row band, at most 64 splits and four waves."""
    sp = lambda t, ctx, w=0: la.lib().lfm3a_prefill_splits(t, 32, ctx, w, 148)
    assert sp(32768, 0) == 1 and sp(1184, 100000) == 1
    assert sp(32, 131072) == 37          # 8 CTAs x 37 = 296: one wave
    assert sp(512, 131072) == 9          # 128 CTAs x 9 = 1152: four nearly full waves (cap: four waves)
    assert sp(1024, 131072) == 1         # 256 CTAs: splitting gains nothing within four waves
    assert sp(64, 20000) == 18           # 16 x 18 = 288
    assert sp(200, 1000) == 2            # 17 tiles in the first band: at most 2 splits of >= 8
    assert sp(32, 100) == 1              # too few tiles to split
    assert sp(32, 10 ** 6, 300) == 1     # a 300-token window: bands of 6 tiles
    assert sp(32, 10 ** 6, 4096) == 8    # 4127 keys: 65 tiles, at most 8 splits
    assert la.lib().lfm3a_prefill_splits(-1, 32, 0, 0, 148) == la.EINVAL


def test_ring_table(la):
    t = la.ring_table(6, 20)
    assert list(t) == [b % 6 for b in range(20)]
    with pytest.raises(la.LFM3AError):
        la.ring_table(5, 4)   # whole 64-token int8 V blocks: an even ring


def test_g128_sizes_and_checks(la):
    lib = la.lib()
    assert lib.lfm3a_g128_packed_bytes(300, 384) == 3 * 3 * 16384
    assert lib.lfm3a_g128_scale_bytes(300, 384) == 3 * 384 * 4
    assert lib.lfm3a_g128_workspace_bytes(300, 384) == 3 * 3 * 16384 + 3 * 384 * 4
    assert lib.lfm3a_g128_packed_bytes(300, 100) == la.EINVAL
    assert lib.lfm3a_g128_packed_bytes(0, 128) == la.EINVAL
    # argument checks answer before anything reaches the device
    assert lib.lfm3a_g128_gemm(None, None, None, None, 4, 4, 128, None, 0, None, 0, None) == la.EINVAL
    assert lib.lfm3a_g128_gemm(None, None, None, None, 4, 4, 96, None, 0, None, 0, None) == la.EINVAL
    assert lib.lfm3a_g128_quantize(None, 128, 4, 128, 0, None, None, None) == la.EINVAL
    assert lib.lfm3a_g128_pack(None, 128, None, 1, 4, 128, None, None, None) == la.EINVAL
    ws = ctypes.create_string_buffer(64)
    addr = (ctypes.addressof(ws) + 15) & ~15
    assert lib.lfm3a_g128_linear(None, 128, 4, 0, None, None, 4, 128, None, 0, None, 4, addr, 16, None) == la.EWORKSPACE


def test_head_dim_128_host_logic(la):
    """The reference geometry (16/4/128) runs one CTA per SM: half the verify splits of head_dim 64 at the same
    kv-head count, and prefill workspaces sized with head_dim + 2 floats per partial row."""
    lib = la.lib()
    l64, l128 = la.layout(0, 4, 64), la.layout(0, 4, 128)
    s64 = lib.lfm3a_verify_splits(ctypes.byref(l64), 131072, 8, 0, 148)
    s128 = lib.lfm3a_verify_splits(ctypes.byref(l128), 131072, 8, 0, 148)
    assert (s64, s128) == (74, 37)
    # past 16 tokens head_dim 128 is refused, so the split count follows the two-per-SM rule
    assert lib.lfm3a_verify_splits(ctypes.byref(l128), 131072, 17, 0, 148) == 74
    assert lib.lfm3a_verify_workspace_bytes(8, 16, 128, 37) == 8 * 16 * 37 * 130 * 4
    # a 64-token chunk of 16 query heads never fills a wave: the workspace covers its long-context splits
    assert lib.lfm3a_prefill_workspace_bytes(64, 16, 128) > 0
    assert lib.lfm3a_prefill_workspace_bytes(64, 16, 96) == 0
    assert lib.lfm3a_prefill_workspace_bytes(64, 16, 128) % (64 * 16 * 130 * 4) == 0


def test_refusals_come_before_any_launch(la):
    """Argument faults that only show once the split count is known are refused before the first launch: a
    gather over a context of one key tile (no combine to scatter from), and a verify round whose workspace is
    too small (the drafts would otherwise already be appended). On this CPU-only host a launch would fail
    with LFM3A_ECUDA, so the codes below also show that nothing was launched."""
    lib = la.lib()
    good = la.KvView(64, 64, 10, la.layout(0, 8, 64))
    half = la.KvView(64, 64, 10, la.layout(0, 4, 64))   # one rank of two under the kv-head plan
    peers = (ctypes.c_void_p * 2)(64, 128)
    # 40 cached tokens + 8 drafts: one 128-key tile.
    rc = lib.lfm3a_verify_attention_gather(ctypes.byref(half), 64, 8, 16, 40, 0, None, peers, 2, 0, 64, 1 << 20, 1,
                                           None)
    assert rc == la.ENOTSUP
    assert b"gather" in lib.lfm3a_last_error()
    # 1000 cached tokens, 16 drafts, 4 splits: the partials need 16 * 32 * 4 * 66 * 4 bytes.
    rc = lib.lfm3a_verify_round(ctypes.byref(good), 64, 64, 0, None, None, 64, 16, 32, 1000, 0, None, 64, 64, 16, 4,
                                None)
    assert rc == la.EWORKSPACE
    assert lib.lfm3a_set_wait_limit  # exported; setting it needs a device


def test_synth_head_slices_match_full_draw(synth):
    """A rank of the kv-head plan draws only its heads (verify_case_heads); the values are the full draw's."""
    full = synth.verify_case(9, 700, 16)
    for h0, h1 in [(0, 8), (0, 1), (3, 5), (7, 8)]:
        part = synth.verify_case_heads(9, 700, 16, h0, h1)
        for k in ("K", "V", "newK", "newV"):
            assert np.array_equal(part[k].view(np.uint16), full[k][:, h0:h1].view(np.uint16)), k
        assert np.array_equal(part["Q"].view(np.uint16), full["Q"][:, 4 * h0:4 * h1].view(np.uint16))


def test_committed_cubin_is_an_sm100a_image(la):
    """The committed kernel image that lfm3a_load_cubin takes: an ELF object for CUDA (e_machine 190)."""
    data = la.CUBIN_PATH.read_bytes()
    assert data[:4] == b"\x7fELF" and len(data) > 100000
    assert int.from_bytes(data[18:20], "little") == 190
    assert la.lib().lfm3a_load_cubin(None, 0) == la.EINVAL
