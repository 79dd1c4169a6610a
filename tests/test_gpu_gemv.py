"""GPU parity of the int4 GEMV and the affine quantizer against the oracle
(bit-exact), through the C ABI."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(dev)
    return torch.from_numpy(a).to(dev)


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _scale_view(t, sd):
    return t.view(torch.float16 if sd == 0 else torch.bfloat16)


@pytest.mark.parametrize("k", [256, 768, 1024, 2048, 4096])
@pytest.mark.parametrize("sd", [0, 1])
def test_gemv_bitexact(cuda, k, sd):
    from rec_b200 import ops

    rng = np.random.default_rng(1000 + k + sd)
    n = 4096 + 2 * 37  # rows not a multiple of the stage size
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scales, biases = oracle.quantize(w, 4, sd)
    x = oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    y = ops.gemv_int4(_t(codes, cuda), _scale_view(_t(scales, cuda), sd), _scale_view(_t(biases, cuda), sd),
                      _t(x, cuda).view(torch.bfloat16))
    torch.cuda.synchronize()
    ref = oracle.gemv(codes, scales, biases, x, sd)
    got = _u16(y)
    assert np.array_equal(got, ref), np.flatnonzero(got != ref)[:10]


@pytest.mark.parametrize("k", [2048, 4096])
def test_gemv_fused_rmsnorm_bitexact(cuda, k):
    from rec_b200 import ops

    rng = np.random.default_rng(7 + k)
    n = 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scales, biases = oracle.quantize(w, 4, 0)
    h = oracle.f32_to_bf16((rng.standard_normal(k) * 2).astype(np.float32))
    nw = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(k)).astype(np.float32))
    y = ops.gemv_int4(_t(codes, cuda), _scale_view(_t(scales, cuda), 0), _scale_view(_t(biases, cuda), 0),
                      _t(h, cuda).view(torch.bfloat16), norm_weight=_t(nw, cuda).view(torch.bfloat16), eps=1e-6)
    xn = oracle.rmsnorm(h, nw, 1e-6)
    ref = oracle.gemv(codes, scales, biases, xn, 0)
    assert np.array_equal(_u16(y), ref)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("sd", [0, 1])
def test_quantize_bitexact(cuda, bits, sd):
    from rec_b200 import ops

    rng = np.random.default_rng(bits * 10 + sd)
    w = (rng.standard_normal((300, 512)) * 0.02).astype(np.float32)
    w[0, :64] = 0.0
    w[1, :64] = -2.5
    w[2, :64] = np.linspace(-1, 1, 64)
    w[3] = rng.standard_normal(512).astype(np.float32) * 50
    codes, scales, biases = ops.quantize_affine(torch.from_numpy(w).to(cuda), bits,
                                                torch.float16 if sd == 0 else torch.bfloat16)
    rc, rs, rb = oracle.quantize(w, bits, sd)
    assert np.array_equal(codes.cpu().numpy().view(np.uint32), rc)
    assert np.array_equal(_u16(scales), rs)
    assert np.array_equal(_u16(biases), rb)
