"""The W8A8 prefill GEMM (kernels/gemm.hip) on the GPU, through the C ABI, against the oracle: the weight packer,
the activation quantiser (plain and gated) and the group-scaled int8 GEMM are bit-exact, on ragged shapes, with a
residual, across the persistent tile walk, and on sampled rows of the model's largest shape."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rand_weights(rng, rows, k):
    w = np.clip(np.rint(rng.normal(size=(rows, k)) * 40.0), -127, 127).astype(np.int8)
    ws = (np.abs(rng.normal(size=(rows, k // 128))) * 0.01 + 1e-3).astype(np.float16).astype(np.float32)
    return w, ws


def dev(torch, a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def unpack(orc, op):
    return orc.g128_unpack(op.data.cpu().numpy(), op.scales.cpu().numpy(), op.rows, op.k)


def bits(a):
    return np.asarray(a).view(np.uint16)


@pytest.mark.parametrize("rows,k", [(300, 384), (1, 128), (128, 2048)])
def test_pack_matches_layout(la, orc, cuda, rows, k):
    import torch

    rng = np.random.default_rng(rows + k)
    w, ws = rand_weights(rng, rows, k)
    op = la.G128Operand.pack(dev(torch, w, cuda), dev(torch, ws, cuda))
    torch.cuda.synchronize()
    packed, sp = orc.g128_pack(w, ws)
    assert np.array_equal(op.data.cpu().numpy(), packed)
    assert np.array_equal(op.scales.cpu().numpy().view(np.uint32), sp.reshape(-1).view(np.uint32))


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("rows,k,stride", [(200, 384, 384), (129, 256, 520), (7, 128, 256), (1, 2048, 2048)])
def test_quantize_bit_exact(la, orc, synth, cuda, gated, rows, k, stride):
    import torch

    width = 2 * k if gated else k
    stride = max(stride, width)
    x = synth.Stream(7 + rows).normal_f16((rows, stride)) * np.float16(3.0)
    x[0, :128] = 0                       # an all-zero group: scale 1
    if gated and rows > 2:
        x[1, :k] = np.float16(-100.0)    # e^-x past the upper clamp
        x[2, :k] = np.float16(95.0)      # past the lower clamp
    op = la.G128Operand.quantize(dev(torch, x, cuda), k, gated=gated)
    torch.cuda.synchronize()
    q, sc = unpack(orc, op)
    wq, wsc = orc.g128_quantize(x, k, gated=gated)
    assert np.array_equal(q, wq)
    assert np.array_equal(sc.view(np.uint32), wsc.view(np.uint32))
    # padding rows of the last tile: zero bytes, scale 1
    full_q, _ = orc.g128_unpack(op.data.cpu().numpy(), op.scales.cpu().numpy(), (rows + 127) // 128 * 128, k)
    assert not full_q[rows:].any()


@pytest.mark.parametrize("rows,outputs,k,resid", [(200, 72, 384, False), (200, 72, 384, True), (130, 600, 256, True),
                                                  (1, 40, 128, False), (2048, 4096, 128, False),
                                                  (257, 3088, 2048, True)])
def test_gemm_bit_exact(la, orc, synth, cuda, rows, outputs, k, resid):
    import torch

    rng = np.random.default_rng(rows * 7 + outputs)
    w, ws = rand_weights(rng, outputs, k)
    x = synth.Stream(rows + outputs).normal_f16((rows, k))
    r = synth.Stream(rows + outputs + 1).normal_f16((rows, outputs)) if resid else None
    b = la.G128Operand.pack(dev(torch, w, cuda), dev(torch, ws, cuda))
    a = la.G128Operand.quantize(dev(torch, x, cuda), k)
    out = la.g128_gemm(a, b, residual=None if r is None else dev(torch, r, cuda))
    torch.cuda.synchronize()
    qa, sa = unpack(orc, a)
    want = orc.g128_gemm(qa, sa, w, ws, residual=r)
    got = out.cpu().numpy()
    assert np.array_equal(bits(got), bits(want)), f"{np.count_nonzero(bits(got) != bits(want))} differ"


def test_linear_gated_strided_out(la, orc, synth, cuda):
    """The down projection: silu(gate) * up quantised and multiplied in one call, into a strided output."""
    import torch

    rows, k, outputs = 300, 768, 264
    rng = np.random.default_rng(11)
    w, ws = rand_weights(rng, outputs, k)
    x = synth.Stream(12).normal_f16((rows, 2 * k))
    b = la.G128Operand.pack(dev(torch, w, cuda), dev(torch, ws, cuda))
    big = torch.full((rows, outputs + 40), float("nan"), dtype=torch.float16, device=cuda)
    out = big[:, 8:8 + outputs]
    la.g128_linear(dev(torch, x, cuda), b, gated=True, out=out)
    torch.cuda.synchronize()
    qa, sa = orc.g128_quantize(x, k, gated=True)
    want = orc.g128_gemm(qa, sa, w, ws)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    assert torch.isnan(big[:, :8]).all() and torch.isnan(big[:, 8 + outputs:]).all()   # nothing outside the view


def test_gemm_full_size_sampled_rows(la, orc, synth, cuda):
    """w13 at the reference's long-prompt chunk: 7680 tokens x 2048 inputs -> 15360 outputs; the oracle checks 24
    rows spread over the tiles (all outputs), bit for bit, and two consecutive calls give identical bytes."""
    import torch

    rows, k, outputs = 7680, 2048, 15360
    g = torch.Generator(device=cuda).manual_seed(3)
    x = (torch.randn((rows, k), generator=g, device=cuda) * 2).half()
    w = torch.randint(-127, 128, (outputs, k), generator=g, device=cuda, dtype=torch.int32).to(torch.int8)
    ws = (torch.rand((outputs, k // 128), generator=g, device=cuda) * 0.01 + 1e-3).half().float()
    b = la.G128Operand.pack(w, ws)
    out = la.g128_linear(x, b)
    out2 = la.g128_linear(x, b)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    sel = np.unique(np.concatenate([np.arange(0, rows, 331), [127, 128, rows - 1]]))
    xs = x[sel].cpu().numpy()
    qa, sa = orc.g128_quantize(xs, k)
    want = orc.g128_gemm(qa, sa, w.cpu().numpy(), ws.cpu().numpy())
    assert np.array_equal(bits(out[sel].cpu().numpy()), bits(want))
