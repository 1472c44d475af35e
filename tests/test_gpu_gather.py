"""The kv-head plan's exchange on one GPU: two ranks emulated in one process (their gather regions both local),
each verifying its 4 kv heads and scattering its output into both regions. Per call the ranks' combines run
before either waits (one stream), so no kernel waits on another that has not run. Three calls in a row
alternate the regions' halves; every gathered output must match the oracle's verify of all 8 heads
(4e-3 of the RMS beyond half an fp16 ulp)."""
import numpy as np
import pytest

from shard import head_range, query_head_range

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def rel_err(got, want):
    want = want.astype(np.float64)
    rms = float(np.sqrt(np.mean(want ** 2)))
    half_ulp = 0.5 * np.abs(np.spacing(want.astype(np.float16))).astype(np.float64)
    return float(np.max(np.clip(np.abs(got.astype(np.float64) - want) - half_ulp, 0.0, None))) / rms


@pytest.mark.parametrize("splits", [0, 7, 200])
def test_heads_gather_two_emulated_ranks(la, orc, synth, cuda, splits):
    """splits 0: the library's count; 7; 200: more splits than the narrow combine holds (the row-per-block
    combine scatters)."""
    import torch

    ctx, m, world = 6000, 16, 2
    c = synth.verify_case(61, ctx, m)
    K = np.concatenate([c["K"], c["newK"]])
    V = np.concatenate([c["V"], c["newV"]])
    rows = m * 16
    regions = [la.GatherGroup.alloc_region(world, rows, 64) for _ in range(world)]
    try:
        groups = [la.GatherGroup(world, r, rows, 64, regions=regions) for r in range(world)]
        caches = []
        for r in range(world):
            h0, h1 = head_range(world, r, 8)
            cache = la.LayerCache(la.MODE_F16, h1 - h0, 64, ctx + m + 64, device=cuda)
            cache.append(dev(K[:, h0:h1], cuda), dev(V[:, h0:h1], cuda), 0)
            caches.append(cache)
        s = synth.Stream(62)
        for call in range(3):
            Q = c["Q"] if call == 0 else s.normal_f16((m, 32, 64))
            for r in range(world):
                q0, q1 = query_head_range(world, r, 8, 32)
                groups[r].verify(caches[r], dev(Q[:, q0:q1], cuda), ctx, splits=splits)
            want = orc.verify(Q, K, V, ctx)
            for r in range(world):
                out = torch.zeros((world, m, 16, 64), dtype=torch.float16, device=cuda)
                groups[r].wait(out)
                la.sync()
                got = out.permute(1, 0, 2, 3).reshape(m, 32, 64).float().cpu().numpy()
                assert rel_err(got, want) < 4e-3, (call, r)
    finally:
        for reg in regions:
            la.lib().lfm3a_gather_region_free(reg)


def test_gather_wait_runs_out_and_recovers(la, orc, synth, cuda):
    """Failure detection without a GPU fault (the bounded Wait of internal/kfd/queue.go:292-310): of two emulated
    ranks only rank 0 verifies in one call, so rank 1's slice never lands. Each region's wait, with the limit set
    to 20 ms, gives up, raises the device error word and returns; lfm3a_sync reports LFM3A_EDEVICE. With the
    default limit restored the ranks stay in step: the next call, made by both, gathers the right output."""
    import torch

    ctx, m, world = 3000, 8, 2
    c = synth.verify_case(63, ctx, m)
    K = np.concatenate([c["K"], c["newK"]])
    V = np.concatenate([c["V"], c["newV"]])
    rows = m * 16
    regions = [la.GatherGroup.alloc_region(world, rows, 64) for _ in range(world)]
    try:
        groups = [la.GatherGroup(world, r, rows, 64, regions=regions) for r in range(world)]
        caches, qs = [], []
        for r in range(world):
            h0, h1 = head_range(world, r, 8)
            q0, q1 = query_head_range(world, r, 8, 32)
            cache = la.LayerCache(la.MODE_F16, h1 - h0, 64, ctx + m + 64, device=cuda)
            cache.append(dev(K[:, h0:h1], cuda), dev(V[:, h0:h1], cuda), 0)
            caches.append(cache)
            qs.append(dev(c["Q"][:, q0:q1], cuda))
        la.sync()
        la.set_wait_limit(20_000_000)
        try:
            groups[0].verify(caches[0], qs[0], ctx)      # rank 1 never verifies in this call
            for r in range(world):
                groups[r].wait(None)
            with pytest.raises(la.LFM3AError) as err:
                la.sync(timeout_ms=10000)
            assert err.value.code == la.EDEVICE
        finally:
            la.set_wait_limit(0)
        la.sync()                                        # the error word was cleared
        for r in range(world):
            groups[r].verify(caches[r], qs[r], ctx)
        want = orc.verify(c["Q"], K, V, ctx)
        for r in range(world):
            out = torch.zeros((world, m, 16, 64), dtype=torch.float16, device=cuda)
            groups[r].wait(out)
            la.sync()
            got = out.permute(1, 0, 2, 3).reshape(m, 32, 64).float().cpu().numpy()
            assert rel_err(got, want) < 4e-3, r
    finally:
        for reg in regions:
            la.lib().lfm3a_gather_region_free(reg)


def test_round_gather_two_emulated_ranks(la, orc, synth, cuda):
    """lfm3a_verify_round_gather: each emulated rank appends its heads' drafts inside the attention kernel and
    scatters its output; two rounds in a row (the second over the first's kept drafts); the gathered output against
    the oracle's verify of all 8 heads, and the drafts' cache bytes bit-exact."""
    import torch

    ctx, m, world = 5000, 16, 2
    c = synth.verify_case(64, ctx, m)
    rope_np = la.rope_table(1e6, 1.0, 64, ctx + 2 * m + 1)
    rope = dev(rope_np.view(np.float16), cuda)
    rows = m * 16
    regions = [la.GatherGroup.alloc_region(world, rows, 64) for _ in range(world)]
    try:
        groups = [la.GatherGroup(world, r, rows, 64, regions=regions) for r in range(world)]
        caches = []
        for r in range(world):
            h0, h1 = head_range(world, r, 8)
            cache = la.LayerCache(la.MODE_F16, h1 - h0, 64, ctx + 2 * m + 64, device=cuda)
            cache.append(dev(c["K"][:, h0:h1], cuda), dev(c["V"][:, h0:h1], cuda), 0)
            caches.append(cache)
        K, V = c["K"], c["V"]
        s = synth.Stream(65)
        length = ctx
        for rnd in range(2):
            nk, nv = (c["newK"], c["newV"]) if rnd == 0 else (s.normal_f16((m, 8, 64)), s.normal_f16((m, 8, 64)))
            Q = c["Q"] if rnd == 0 else s.normal_f16((m, 32, 64))
            for r in range(world):
                h0, h1 = head_range(world, r, 8)
                q0, q1 = query_head_range(world, r, 8, 32)
                groups[r].verify_round(caches[r], dev(nk[:, h0:h1], cuda), dev(nv[:, h0:h1], cuda),
                                       dev(Q[:, q0:q1], cuda), length, rope=rope)
            kn, vn = orc.kv_append_f16(nk, nv, length, rope=rope_np.view(np.float16))
            K = np.concatenate([K[:length], kn])
            V = np.concatenate([V[:length], vn])
            want = orc.verify(Q, K, V, length)
            for r in range(world):
                out = torch.zeros((world, m, 16, 64), dtype=torch.float16, device=cuda)
                groups[r].wait(out)
                la.sync()
                got = out.permute(1, 0, 2, 3).reshape(m, 32, 64).float().cpu().numpy()
                assert rel_err(got, want) < 4e-3, (rnd, r)
            for r in range(world):
                h0, h1 = head_range(world, r, 8)
                caches[r].truncate(length + 5)
                logical = caches[r].logical(length + 5)
                assert np.array_equal(logical["K"][length:], K[length:length + 5, h0:h1].view(np.uint16))
            length += 5
    finally:
        for reg in regions:
            la.lib().lfm3a_gather_region_free(reg)


def test_gather_head_dim_128(la, orc, synth, cuda):
    """The exchange at the reference model's 16/4/128 geometry: two emulated ranks of two kv heads each, rounds with
    the drafts' append fused into the attention kernel, the gathered output against the oracle's verify."""
    import torch

    ctx, m, world, d = 7000, 9, 2, 128
    c = synth.verify_case(66, ctx, m, q_heads=16, kv_heads=4, head_dim=d)
    rope_np = la.rope_table(1e6, 0.5, d, ctx + m + 1)
    rows = m * 8
    regions = [la.GatherGroup.alloc_region(world, rows, d) for _ in range(world)]
    try:
        groups = [la.GatherGroup(world, r, rows, d, regions=regions) for r in range(world)]
        for r in range(world):
            h0, h1 = head_range(world, r, 4)
            q0, q1 = query_head_range(world, r, 4, 16)
            cache = la.LayerCache(la.MODE_F16, h1 - h0, d, ctx + m + 64, device=cuda)
            cache.append(dev(c["K"][:, h0:h1], cuda), dev(c["V"][:, h0:h1], cuda), 0)
            groups[r].verify_round(cache, dev(c["newK"][:, h0:h1], cuda), dev(c["newV"][:, h0:h1], cuda),
                                   dev(c["Q"][:, q0:q1], cuda), ctx, rope=dev(rope_np.view(np.float16), cuda))
        kn, vn = orc.kv_append_f16(c["newK"], c["newV"], ctx, rope=rope_np.view(np.float16))
        want = orc.verify(c["Q"], np.concatenate([c["K"], kn]), np.concatenate([c["V"], vn]), ctx)
        for r in range(world):
            out = torch.zeros((world, m, 8, d), dtype=torch.float16, device=cuda)
            groups[r].wait(out)
            la.sync()
            got = out.permute(1, 0, 2, 3).reshape(m, 16, d).float().cpu().numpy()
            assert rel_err(got, want) < 4e-3, r
    finally:
        for reg in regions:
            la.lib().lfm3a_gather_region_free(reg)
