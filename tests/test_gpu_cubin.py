"""The committed sm_100a cubin loaded through the CUDA driver API (lfm3a_load_cubin): the config-1 smoke round
(append with RoPE, verify attention, rollback) and an exact prefill run from the module's kernels, checked against
the oracle as the smoke does (cache bytes bit-exact, attention within its tolerances), and every launch counted by
the module. Unloading goes back to the library's own kernels."""
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


def test_kernels_from_the_committed_cubin(la, orc, synth, cuda):
    import __graft_entry__ as entry

    la.sync()
    assert la.cubin_launches() == -1
    la.load_cubin()
    try:
        assert la.cubin_launches() == 0
        entry.smoke()   # raises on any mismatch against the oracle
        after_smoke = la.cubin_launches()
        assert after_smoke >= 4   # two appends, verify + combine, the rollback's re-quantisation
        c = synth.prefill_case(71, 700)
        cache = la.LayerCache(la.MODE_F16, 8, 64, 800, device=cuda)
        cache.append(dev(c["K"], cuda), dev(c["V"], cuda), 0)
        out = cache.prefill(dev(c["Q"], cuda), 0, exact=True)
        la.sync()
        assert la.cubin_launches() > after_smoke
        want = orc.prefill_exact(c["Q"], 0, c["K"], c["V"])
        assert rel_err(out.float().cpu().numpy(), want) < 4e-3
        with pytest.raises(la.LFM3AError):
            la.load_cubin()   # one module per device
    finally:
        la.unload_cubin()
    assert la.cubin_launches() == -1
